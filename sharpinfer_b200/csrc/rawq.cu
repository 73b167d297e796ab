// Q4_0, Q2_K, Q3_K and Q5_K weights: stored on the device in their GGUF
// block layout (no re-ordering), dequantised bit-exactly, multiplied by f32
// activations in a warp-per-row matvec and pre-dequantised to f16 for the
// prefill GEMM.
//
// Layouts are GGML's, the ones GGUF files hold (pinned to gguf-py by the
// golden vectors): Q4_0 [f16 d][qs 16]; Q2_K [scales 16][qs 64][f16 d]
// [f16 dmin]; Q3_K [hmask 32][qs 64][scales 12][f16 d]; Q5_K [f16 d][f16 dmin]
// [scales 12][qh 32][qs 128].  The arithmetic of each element is the
// reference's (Quantization.cs: Q4_0 :71-83 ((q & 15) - 8) * d; Q2_K :176-197
// (d * sc) * q - dmin * m; Q3_K :205-267 (d * (sc - 32)) * (q2 + hb); Q5_K
// :322-356 (d * sc) * q - dmin * m), each product and difference rounded once.
//
// A unit is 256 consecutive elements of a row (8 Q4_0 blocks, or one K-quant
// superblock); lane L of a warp owns its elements 8L .. 8L + 7.
#include "common.cuh"

namespace si {
namespace {

__device__ __forceinline__ float hf(const uint8_t* p) {
  return __half2float(__ushort_as_half((unsigned short)(p[0] | (p[1] << 8))));
}

// The 8 values of elements 8 lane .. 8 lane + 7 of a unit.
template <int QT>
__device__ __forceinline__ void decode8(const uint8_t* __restrict__ u, int lane, float (&v)[8]) {
  if (QT == SI_Q4_0) {
    const uint8_t* b = u + (lane >> 2) * 18;  // block lane / 4, quarter lane % 4
    const int part = lane & 3;
    const float d = hf(b);
    const uint8_t* q = b + 2 + 8 * (part & 1);
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const int nib = part < 2 ? (q[i] & 0xF) : (q[i] >> 4);
      v[i] = __fmul_rn((float)(nib - 8), d);
    }
  } else if (QT == SI_Q2_K) {
    const int n = lane >> 4, s = (lane >> 2) & 3, h = (lane >> 1) & 1, l0 = 8 * (lane & 1);
    const uint8_t sc = u[8 * n + 2 * s + h];
    const float dl = __fmul_rn(hf(u + 80), (float)(sc & 0xF)), ml = __fmul_rn(hf(u + 82), (float)(sc >> 4));
    const uint8_t* q = u + 16 + 32 * n + 16 * h + l0;
#pragma unroll
    for (int i = 0; i < 8; i++) v[i] = __fsub_rn(__fmul_rn(dl, (float)((q[i] >> (2 * s)) & 3)), ml);
  } else if (QT == SI_Q3_K) {
    const int n = lane >> 4, j = (lane >> 2) & 3, h = (lane >> 1) & 1, l0 = 8 * (lane & 1);
    const int idx = 8 * n + 2 * j + h, i4 = idx & 3;  // 6-bit scale idx of 16
    const uint8_t* raw = u + 96;
    const int lo = idx < 8 ? (raw[idx] & 0xF) : (raw[idx - 8] >> 4);
    const int hi = (raw[8 + i4] >> (2 * (idx >> 2))) & 3;
    const float dl = __fmul_rn(hf(u + 108), (float)((lo | (hi << 4)) - 32));
    const uint8_t* q = u + 32 + 32 * n + 16 * h + l0;
    const uint8_t* hm = u + 16 * h + l0;
    const int bit = 4 * n + j;
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const int q2 = (q[i] >> (2 * j)) & 3, hb = ((hm[i] >> bit) & 1) ? 0 : -4;
      v[i] = __fmul_rn(dl, (float)(q2 + hb));
    }
  } else {  // SI_Q5_K
    const int j = lane >> 3, half = (lane >> 2) & 1, l0 = 8 * (lane & 3);
    const int s = 2 * j + half;
    const uint8_t* sc = u + 4;
    uint32_t scv, mnv;  // GetScaleMinK4 (Quantization.cs:302-314)
    if (s < 4) {
      scv = sc[s] & 63;
      mnv = sc[s + 4] & 63;
    } else {
      scv = (sc[s + 4] & 0xF) | ((sc[s - 4] >> 6) << 4);
      mnv = (sc[s + 4] >> 4) | ((sc[s] >> 6) << 4);
    }
    const float d1 = __fmul_rn(hf(u), (float)scv), m1 = __fmul_rn(hf(u + 2), (float)mnv);
    const uint8_t* qh = u + 16 + l0;
    const uint8_t* qs = u + 48 + 32 * j + l0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const int q = (half ? (qs[i] >> 4) : (qs[i] & 0xF)) + (((qh[i] >> s) & 1) << 4);
      v[i] = __fsub_rn(__fmul_rn(d1, (float)q), m1);
    }
  }
}

template <int QT>
struct RawInfo;
template <> struct RawInfo<SI_Q4_0> { static constexpr int UB = 8 * 18; };
template <> struct RawInfo<SI_Q2_K> { static constexpr int UB = 84; };
template <> struct RawInfo<SI_Q3_K> { static constexpr int UB = 110; };
template <> struct RawInfo<SI_Q5_K> { static constexpr int UB = 176; };

// out[r][c] (f32, or f16 rounded once from the f32 value); one warp per unit.
template <int QT, typename T>
__global__ void __launch_bounds__(256) k_dequant_raw(const uint8_t* __restrict__ W, int64_t units, T* __restrict__ out) {
  const int64_t u = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (u >= units) return;
  float v[8];
  decode8<QT>(W + u * RawInfo<QT>::UB, lane, v);
  T* o = out + u * 256 + 8 * lane;
#pragma unroll
  for (int i = 0; i < 8; i++) {
    if constexpr (sizeof(T) == 4) o[i] = v[i];
    else o[i] = __float2half_rn(v[i]);
  }
}

// y[b][r] = sum_c W[r][c] x[b][c]: one warp per row (8 rows per CTA), each
// lane decoding its 8 elements of every unit once for all B vectors.
template <int QT, int B>
__global__ void __launch_bounds__(256) k_qmv_raw(const uint8_t* __restrict__ W, int64_t rows, int nunit,
                                                 const float* __restrict__ x, float* __restrict__ y) {
  const int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const int K = nunit * 256;
  const uint8_t* wr = W + r * (int64_t)nunit * RawInfo<QT>::UB;
  float acc[B];
#pragma unroll
  for (int b = 0; b < B; b++) acc[b] = 0.f;
  for (int u = 0; u < nunit; u++) {
    float v[8];
    decode8<QT>(wr + (int64_t)u * RawInfo<QT>::UB, lane, v);
#pragma unroll
    for (int b = 0; b < B; b++) {
      const float4* xp = (const float4*)(x + (int64_t)b * K + 256 * u + 8 * lane);
      const float4 x0 = __ldg(xp), x1 = __ldg(xp + 1);
      acc[b] = fmaf(v[0], x0.x, acc[b]);
      acc[b] = fmaf(v[1], x0.y, acc[b]);
      acc[b] = fmaf(v[2], x0.z, acc[b]);
      acc[b] = fmaf(v[3], x0.w, acc[b]);
      acc[b] = fmaf(v[4], x1.x, acc[b]);
      acc[b] = fmaf(v[5], x1.y, acc[b]);
      acc[b] = fmaf(v[6], x1.z, acc[b]);
      acc[b] = fmaf(v[7], x1.w, acc[b]);
    }
  }
#pragma unroll
  for (int b = 0; b < B; b++) {
    const float s = warp_sum(acc[b]);
    if (lane == 0) y[(int64_t)b * rows + r] = s;
  }
}

template <int QT>
int launch_qmv_raw_b(cudaStream_t s, const si_weight* w, const float* x, float* y, int B) {
  const int nunit = (int)(w->cols / 256);
  const unsigned grid = (unsigned)((w->rows + 7) / 8);
  switch (B) {
#define SI_RAW_B(BB) \
  case BB: k_qmv_raw<QT, BB><<<grid, 256, 0, s>>>((const uint8_t*)w->dev, w->rows, nunit, x, y); break;
    SI_RAW_B(1) SI_RAW_B(2) SI_RAW_B(3) SI_RAW_B(4) SI_RAW_B(5) SI_RAW_B(6) SI_RAW_B(7) SI_RAW_B(8)
    SI_RAW_B(9) SI_RAW_B(10) SI_RAW_B(11) SI_RAW_B(12) SI_RAW_B(13) SI_RAW_B(14) SI_RAW_B(15) SI_RAW_B(16)
#undef SI_RAW_B
    default: SI_FAIL(SI_ERR_INVALID, "qmatvec: batch %d outside 1..16", B);
  }
  SI_CUDA(cudaGetLastError());
  return SI_OK;
}

template <typename T>
int launch_dequant_raw_t(cudaStream_t s, const si_weight* w, T* out) {
  const int64_t units = w->rows * (w->cols / 256);
  const unsigned grid = (unsigned)((units + 7) / 8);
  const uint8_t* W = (const uint8_t*)w->dev;
  switch (w->qtype) {
    case SI_Q4_0: k_dequant_raw<SI_Q4_0, T><<<grid, 256, 0, s>>>(W, units, out); break;
    case SI_Q2_K: k_dequant_raw<SI_Q2_K, T><<<grid, 256, 0, s>>>(W, units, out); break;
    case SI_Q3_K: k_dequant_raw<SI_Q3_K, T><<<grid, 256, 0, s>>>(W, units, out); break;
    case SI_Q5_K: k_dequant_raw<SI_Q5_K, T><<<grid, 256, 0, s>>>(W, units, out); break;
    default: SI_FAIL(SI_ERR_UNSUPPORTED, "dequant: quant type %d", w->qtype);
  }
  SI_CUDA(cudaGetLastError());
  return SI_OK;
}

}  // namespace

int launch_qmv_raw(cudaStream_t s, const si_weight* w, const float* x, float* y, int B) {
  if (((uintptr_t)x & 15) || (w->cols % 256)) SI_FAIL(SI_ERR_INVALID, "qmatvec: x must be 16-byte aligned");
  switch (w->qtype) {
    case SI_Q4_0: return launch_qmv_raw_b<SI_Q4_0>(s, w, x, y, B);
    case SI_Q2_K: return launch_qmv_raw_b<SI_Q2_K>(s, w, x, y, B);
    case SI_Q3_K: return launch_qmv_raw_b<SI_Q3_K>(s, w, x, y, B);
    case SI_Q5_K: return launch_qmv_raw_b<SI_Q5_K>(s, w, x, y, B);
    default: SI_FAIL(SI_ERR_UNSUPPORTED, "qmatvec: quant type %d", w->qtype);
  }
}

int launch_dequant_raw(cudaStream_t s, const si_weight* w, float* out) { return launch_dequant_raw_t<float>(s, w, out); }

int launch_dequant_raw_f16(cudaStream_t s, const si_weight* w, __half* out) {
  return launch_dequant_raw_t<__half>(s, w, out);
}

}  // namespace si
