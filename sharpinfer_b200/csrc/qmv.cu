// Fused dequantise + matvec for Q4_K / Q6_K / Q8_0 weights, batch 1..16.
//
// y[b][r] = sum_c W[r][c] x[b][c]  -- the quantised form of
// TensorOps.MatVecMul (src/SharpInfer.Core/Tensors/TensorOps.cs:63-72) with W
// decoded as in Quantization.cs (Q4_K :273-314, Q6_K :362-391, Q8_0 :106-114).
//
// The kernel is bound by HBM: every weight byte is read once.  To keep the
// instruction rate below the byte rate, the multiply-adds run on the tensor
// cores (mma.m16n8k16, f16 inputs, f32 accumulation):
//  * quant codes are small integers and exact in f16; for Q4_K the 6-bit
//    sub-block scale is folded in exactly with one f16 FMA per pair
//    ((1024+q)*sc - 1024*sc = q*sc, exact because q*sc <= 945);
//  * activations are split into f16 hi + lo parts (x*2^e = hi + lo, ~22
//    significant bits) that occupy two MMA columns, so the product keeps
//    f32-level accuracy; batch b uses columns 2(b%4), 2(b%4)+1 of MMA group
//    b/4;
//  * the Q4_K mins term dmin * sum_s m_s * X_s (X_s = sum of x over the 32
//    elements of sub-block s) is one more MMA per block.
// A row tile of 16 rows is one CTA of 8 warps; the warps split the K blocks
// and are reduced through shared memory.
#include "common.cuh"

namespace si {
namespace {

constexpr int QMV_WARPS = 8;

__device__ __forceinline__ float h2f_lo(uint32_t w) {
  return __half2float(__ushort_as_half((unsigned short)(w & 0xFFFF)));
}
__device__ __forceinline__ float h2f_hi(uint32_t w) {
  return __half2float(__ushort_as_half((unsigned short)(w >> 16)));
}

// Split v into f16 hi + lo; part 0 -> hi, 1 -> lo.
__device__ __forceinline__ __half split_part(float v, int part) {
  __half hi = __float2half_rn(v);
  if (part == 0) return hi;
  return __float2half_rn(v - __half2float(hi));
}

__device__ __forceinline__ uint32_t pack2(__half a, __half b) {
  return (uint32_t)__half_as_ushort(a) | ((uint32_t)__half_as_ushort(b) << 16);
}

__device__ __forceinline__ float block_reduce_sum(float v, float* red) {
  v = warp_sum(v);
  int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float r = 0.f;
  for (int i = 0; i < nw; i++) r += red[i];
  return r;
}

__device__ __forceinline__ float block_reduce_max(float v, float* red) {
  v = warp_max(v);
  int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float r = 0.f;
  for (int i = 0; i < nw; i++) r = fmaxf(r, red[i]);
  return r;
}

// ---------------------------------------------------------------------------
// Activation preparation.  One CTA per (padded) batch row.
//   mode 0: v = x
//   mode 1: v = RmsNorm(x) * w   (TensorOps.cs:135-145)
//   mode 2: v = SiLU(x) * x2     (TensorOps.cs:191-195 then :169-185)
// Outputs (lane (g, t) of MMA group mg owns column g = batch 4mg + g/2,
// part g&1 = hi/lo):
//   xfrag [nmg][K/32][32] uint4 = {b01, b23} of k-tiles 2j and 2j+1,
//   xsfrag [nmg][K/256][32] u32 = (X_{2t}, X_{2t+1}) * 2^-5 of the block,
//   xscale[b] = 2^-e where v * 2^e is what the fragments hold.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(512) k_prep(const float* __restrict__ x,
                                              const float* __restrict__ x2,
                                              const float* __restrict__ nw, float eps, int mode,
                                              int K, int B, float* __restrict__ xout,
                                              uint4* __restrict__ xfrag,
                                              uint32_t* __restrict__ xsfrag,
                                              float* __restrict__ xscale) {
  extern __shared__ float sv[];  // K values
  __shared__ float red[32];
  const int b = blockIdx.x, mg = b >> 2, cb = b & 3;
  const bool live = b < B;
  pdl_wait();
  float amax = 0.f;
  if (live) {
    const float* xb = x + (int64_t)b * K;
    float scale = 1.f;
    if (mode == 1) {
      float ss = 0.f;
      for (int k = threadIdx.x; k < K; k += blockDim.x) ss = __fadd_rn(ss, __fmul_rn(xb[k], xb[k]));
      ss = block_reduce_sum(ss, red);
      scale = 1.0f / sqrtf(ss / (float)K + eps);
    }
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
      float v;
      if (mode == 1) {
        v = __fmul_rn(__fmul_rn(xb[k], scale), nw[k]);
      } else if (mode == 2) {
        float gte = xb[k];
        float sl = __fdiv_rn(gte, __fadd_rn(1.0f, expf(-gte)));
        v = __fmul_rn(sl, x2[(int64_t)b * K + k]);
      } else {
        v = xb[k];
      }
      sv[k] = v;
      if (xout) xout[(int64_t)b * K + k] = v;
      amax = fmaxf(amax, fabsf(v));
    }
    amax = block_reduce_max(amax, red);
  }
  __syncthreads();
  int e = 0;
  if (live && amax > 0.f && amax <= 3.0e38f) {
    int E;
    frexpf(amax, &E);  // amax < 2^E
    e = 14 - E;
    e = e < -100 ? -100 : (e > 100 ? 100 : e);
  }
  const float s = ldexpf(1.0f, e);
  if (threadIdx.x == 0) xscale[b] = live ? ldexpf(1.0f, -e) : 0.f;
  const int K32 = K >> 5;
  for (int it = threadIdx.x; it < K32 * 8; it += blockDim.x) {
    int j = it >> 3, part = (it >> 2) & 1, t = it & 3;
    int lane = 8 * cb + 4 * part + t;
    uint4 r = make_uint4(0, 0, 0, 0);
    if (live) {
      uint32_t w[4];
#pragma unroll
      for (int h = 0; h < 2; h++) {
        int base = 32 * j + 16 * h + 2 * t;
        float v0 = sv[base] * s, v1 = sv[base + 1] * s, v2 = sv[base + 8] * s,
              v3 = sv[base + 9] * s;
        w[2 * h] = pack2(split_part(v0, part), split_part(v1, part));
        w[2 * h + 1] = pack2(split_part(v2, part), split_part(v3, part));
      }
      r = make_uint4(w[0], w[1], w[2], w[3]);
    }
    xfrag[((int64_t)mg * K32 + j) * 32 + lane] = r;
  }
  if (xsfrag && (K & 255) == 0) {
    const int K256 = K >> 8;
    const float s5 = s * 0.03125f;  // X * 2^-5 keeps the 32-term sums inside f16 range
    for (int it = threadIdx.x; it < K256 * 8; it += blockDim.x) {
      int bb = it >> 3, part = (it >> 2) & 1, t = it & 3;
      int lane = 8 * cb + 4 * part + t;
      uint32_t r = 0;
      if (live) {
        float X0 = 0.f, X1 = 0.f;
        const float* p0 = sv + 256 * bb + 32 * (2 * t);
        for (int k = 0; k < 32; k++) X0 += p0[k];
        for (int k = 0; k < 32; k++) X1 += p0[32 + k];
        r = pack2(split_part(X0 * s5, part), split_part(X1 * s5, part));
      }
      xsfrag[((int64_t)mg * K256 + bb) * 32 + lane] = r;
    }
  }
  __syncthreads();
  pdl_launch();
}

// ---------------------------------------------------------------------------
// Shared epilogue: reduce the 8 warps' partial sums and write y.
// tg/tg8: rows g and g+8 of the tile, batch 4mg + t.
// ---------------------------------------------------------------------------
template <int NMG, int EPI>
__device__ __forceinline__ void qmv_epilogue(const float (&tg)[NMG], const float (&tg8)[NMG],
                                             const float* __restrict__ xscale, int B, int64_t rows,
                                             float* __restrict__ y) {
  __shared__ float red[QMV_WARPS][NMG][2][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int mg = 0; mg < NMG; mg++) {
    red[warp][mg][0][lane] = tg[mg];
    red[warp][mg][1][lane] = tg8[mg];
  }
  __syncthreads();
  // 2 * NMG * 32 outputs, one per thread.
  const int o = threadIdx.x;
  if (o < 2 * NMG * 32) {
    const int mg = o >> 6, half = (o >> 5) & 1, ln = o & 31;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < QMV_WARPS; w++) v += red[w][mg][half][ln];
    const int gg = ln >> 2, tt = ln & 3;
    const int bt = 4 * mg + tt;
    const int64_t row = (int64_t)blockIdx.x * 16 + gg + 8 * half;
    if (bt < B && row < rows) {
      v *= xscale[bt];
      float* dst = y + (int64_t)bt * rows + row;
      if (EPI == SI_EPI_ADD) *dst += v;
      else *dst = v;
    }
  }
  (void)g;
  (void)t;
}

// ---------------------------------------------------------------------------
// Q4_K
// ---------------------------------------------------------------------------
struct Q4kRegs {
  uint4 h0, h1, q[4];
};

__device__ __forceinline__ void q4k_load(Q4kRegs& r, const uint8_t* tb, int g, int lane) {
  r.h0 = ldg_nc_v4(tb + 16 * g);
  r.h1 = ldg_nc_v4(tb + 16 * (g + 8));
#pragma unroll
  for (int c = 0; c < 4; c++) r.q[c] = ldg_nc_v4(tb + 256 + c * 512 + lane * 16);
}

__device__ __forceinline__ uint32_t sc_half2(uint32_t lo4, uint32_t hi4, int s) {
  // (sc_s, sc_s) as f16x2 for sub-block s of a decoded scale pair of words.
  const uint32_t w = s < 4 ? lo4 : hi4;
  const uint32_t k = s & 3;
  const uint32_t sel = 0x5040u | k | (k << 8);
  return hsub2_u32(prmt(w, 0x64646464u, sel), 0x64006400u);
}

template <int NMG, int EPI>
__global__ void __launch_bounds__(256) k_qmv_q4k(const uint8_t* __restrict__ W, int nblk,
                                                 int64_t rows, const uint4* __restrict__ xfrag,
                                                 const uint32_t* __restrict__ xsfrag,
                                                 const float* __restrict__ xscale, int B,
                                                 float* __restrict__ y) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const uint8_t* tile = W + (int64_t)blockIdx.x * nblk * 2304;
  const int K32 = nblk * 8;
  const uint32_t msel = (t & 1) ? 0x5342u : 0x5140u;
  float tg[NMG], tg8[NMG];
#pragma unroll
  for (int i = 0; i < NMG; i++) tg[i] = tg8[i] = 0.f;

  Q4kRegs cur, nxt;
  int b = warp;
  if (b < nblk) q4k_load(cur, tile + (int64_t)b * 2304, g, lane);
  pdl_wait();
  for (; b < nblk; b += QMV_WARPS) {
    const int bn = b + QMV_WARPS;
    if (bn < nblk) q4k_load(nxt, tile + (int64_t)bn * 2304, g, lane);

    // 6-bit scales and mins of rows g and g+8 (GetScaleMinK4, Quantization.cs:302-314),
    // four per word.
    const uint32_t scl0 = cur.h0.y & 0x3F3F3F3Fu, mnl0 = cur.h0.z & 0x3F3F3F3Fu;
    const uint32_t sch0 = (cur.h0.w & 0x0F0F0F0Fu) | ((cur.h0.y >> 2) & 0x30303030u);
    const uint32_t mnh0 = ((cur.h0.w >> 4) & 0x0F0F0F0Fu) | ((cur.h0.z >> 2) & 0x30303030u);
    const uint32_t scl1 = cur.h1.y & 0x3F3F3F3Fu, mnl1 = cur.h1.z & 0x3F3F3F3Fu;
    const uint32_t sch1 = (cur.h1.w & 0x0F0F0F0Fu) | ((cur.h1.y >> 2) & 0x30303030u);
    const uint32_t mnh1 = ((cur.h1.w >> 4) & 0x0F0F0F0Fu) | ((cur.h1.z >> 2) & 0x30303030u);

    float C[NMG][4], Cm[NMG][4];
#pragma unroll
    for (int mg = 0; mg < NMG; mg++)
#pragma unroll
      for (int i = 0; i < 4; i++) C[mg][i] = Cm[mg][i] = 0.f;

    // mins: A[row][k] = m_k(row) for k < 8, B[k][col] = X_k(col) * 2^-5.
    {
      const uint32_t am0 = hsub2_u32(prmt(t < 2 ? mnl0 : mnh0, 0x64646464u, msel), 0x64006400u);
      const uint32_t am1 = hsub2_u32(prmt(t < 2 ? mnl1 : mnh1, 0x64646464u, msel), 0x64006400u);
#pragma unroll
      for (int mg = 0; mg < NMG; mg++) {
        const uint32_t xs = xsfrag[((int64_t)mg * nblk + b) * 32 + lane];
        mma16816(Cm[mg], am0, am1, 0u, 0u, xs, 0u);
      }
    }
#pragma unroll
    for (int c = 0; c < 4; c++) {
      uint4 xf[NMG][2];
#pragma unroll
      for (int mg = 0; mg < NMG; mg++) {
        const uint4* xp = xfrag + ((int64_t)mg * K32 + (int64_t)b * 8 + 2 * c) * 32 + lane;
        xf[mg][0] = xp[0];
        xf[mg][1] = xp[32];
      }
#pragma unroll
      for (int hs = 0; hs < 2; hs++) {  // sub-block s = 2c + hs
        const int s = 2 * c + hs;
        const uint32_t sg = sc_half2(scl0, sch0, s), sg8 = sc_half2(scl1, sch1, s);
        const uint32_t nsg = hmul2_u32(sg, 0xE400E400u);  // -1024 * sc, exact
        const uint32_t nsg8 = hmul2_u32(sg8, 0xE400E400u);
#pragma unroll
        for (int kk = 0; kk < 2; kk++) {
          const int i = 2 * hs + kk;
          const uint32_t w = i == 0 ? cur.q[c].x : i == 1 ? cur.q[c].y : i == 2 ? cur.q[c].z : cur.q[c].w;
          const uint32_t w8 = w >> 8;
          const uint32_t a0 = hfma2_u32(lop3_and_or(w, 0x000F000Fu, 0x64006400u), sg, nsg);
          const uint32_t a1 = hfma2_u32(lop3_and_or(w, 0x00F000F0u, 0x64006400u), sg8, nsg8);
          const uint32_t a2 = hfma2_u32(lop3_and_or(w8, 0x000F000Fu, 0x64006400u), sg, nsg);
          const uint32_t a3 = hfma2_u32(lop3_and_or(w8, 0x00F000F0u, 0x64006400u), sg8, nsg8);
#pragma unroll
          for (int mg = 0; mg < NMG; mg++) {
            const uint4& xv = xf[mg][hs];
            mma16816(C[mg], a0, a1, a2, a3, kk ? xv.z : xv.x, kk ? xv.w : xv.y);
          }
        }
      }
    }
    const float d0 = h2f_lo(cur.h0.x), dm0 = h2f_hi(cur.h0.x) * 32.f;
    const float d1 = h2f_lo(cur.h1.x) * 0.0625f, dm1 = h2f_hi(cur.h1.x) * 32.f;
#pragma unroll
    for (int mg = 0; mg < NMG; mg++) {
      tg[mg] += d0 * (C[mg][0] + C[mg][1]) - dm0 * (Cm[mg][0] + Cm[mg][1]);
      tg8[mg] += d1 * (C[mg][2] + C[mg][3]) - dm1 * (Cm[mg][2] + Cm[mg][3]);
    }
    if (bn < nblk) cur = nxt;
  }
  pdl_launch();
  qmv_epilogue<NMG, EPI>(tg, tg8, xscale, B, rows, y);
}

// ---------------------------------------------------------------------------
// Q6_K
// ---------------------------------------------------------------------------
struct Q6kRegs {
  uint4 L[4];
  uint2 H[4];
  uint4 s0, s1;
  uint32_t d;
};

__device__ __forceinline__ void q6k_load(Q6kRegs& r, const uint8_t* tb, int g, int lane) {
#pragma unroll
  for (int c = 0; c < 4; c++) {
    r.L[c] = ldg_nc_v4(tb + c * 768 + lane * 16);
    r.H[c] = ldg_nc_v2(tb + c * 768 + 512 + lane * 8);
  }
  r.s0 = ldg_nc_v4(tb + 3072 + 16 * g);
  r.s1 = ldg_nc_v4(tb + 3072 + 16 * (g + 8));
  r.d = *(const uint32_t*)(tb + 3328 + 4 * g);
}

__device__ __forceinline__ float sbyte(uint4 v, int k) {
  const uint32_t w = k < 4 ? v.x : k < 8 ? v.y : k < 12 ? v.z : v.w;
  return (float)(int8_t)((w >> (8 * (k & 3))) & 0xFF);
}

template <int NMG, int EPI>
__global__ void __launch_bounds__(256) k_qmv_q6k(const uint8_t* __restrict__ W, int nblk,
                                                 int64_t rows, const uint4* __restrict__ xfrag,
                                                 const uint32_t* __restrict__ /*unused*/,
                                                 const float* __restrict__ xscale, int B,
                                                 float* __restrict__ y) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2;
  const uint8_t* tile = W + (int64_t)blockIdx.x * nblk * 3360;
  const int K32 = nblk * 8;
  float tg[NMG], tg8[NMG];
#pragma unroll
  for (int i = 0; i < NMG; i++) tg[i] = tg8[i] = 0.f;
  Q6kRegs cur, nxt;
  int b = warp;
  if (b < nblk) q6k_load(cur, tile + (int64_t)b * 3360, g, lane);
  pdl_wait();
  for (; b < nblk; b += QMV_WARPS) {
    const int bn = b + QMV_WARPS;
    if (bn < nblk) q6k_load(nxt, tile + (int64_t)bn * 3360, g, lane);
    const float d0 = h2f_lo(cur.d), d1 = h2f_hi(cur.d) * 0.0625f;
#pragma unroll
    for (int c = 0; c < 4; c++) {
      uint4 xf[NMG][2];
#pragma unroll
      for (int mg = 0; mg < NMG; mg++) {
        const uint4* xp = xfrag + ((int64_t)mg * K32 + (int64_t)b * 8 + 2 * c) * 32 + lane;
        xf[mg][0] = xp[0];
        xf[mg][1] = xp[32];
      }
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int kt = 4 * c + i;
        const uint32_t L = i == 0 ? cur.L[c].x : i == 1 ? cur.L[c].y : i == 2 ? cur.L[c].z : cur.L[c].w;
        const uint32_t Hw = (i < 2 ? cur.H[c].x : cur.H[c].y) >> (2 * (i & 1));
        const uint32_t L8 = L >> 8, H8 = Hw >> 8, Hs = Hw << 8;
        const uint32_t a0 = hsub2_u32(lop3_and_or(L, 0x000F000Fu, lop3_and_or(Hw, 0x00300030u, 0x64006400u)), 0x64206420u);
        const uint32_t a1 = hsub2_u32(lop3_and_or(L, 0x00F000F0u, lop3_and_or(Hw, 0x03000300u, 0x64006400u)), 0x66006600u);
        const uint32_t a2 = hsub2_u32(lop3_and_or(L8, 0x000F000Fu, lop3_and_or(H8, 0x00300030u, 0x64006400u)), 0x64206420u);
        const uint32_t a3 = hsub2_u32(lop3_and_or(L8, 0x00F000F0u, lop3_and_or(Hs, 0x03000300u, 0x64006400u)), 0x66006600u);
        const float f0 = d0 * sbyte(cur.s0, kt), f1 = d1 * sbyte(cur.s1, kt);
#pragma unroll
        for (int mg = 0; mg < NMG; mg++) {
          float Cc[4] = {0.f, 0.f, 0.f, 0.f};
          const uint4& xv = xf[mg][i >> 1];
          mma16816(Cc, a0, a1, a2, a3, (i & 1) ? xv.z : xv.x, (i & 1) ? xv.w : xv.y);
          tg[mg] += f0 * (Cc[0] + Cc[1]);
          tg8[mg] += f1 * (Cc[2] + Cc[3]);
        }
      }
    }
    if (bn < nblk) cur = nxt;
  }
  pdl_launch();
  qmv_epilogue<NMG, EPI>(tg, tg8, xscale, B, rows, y);
}

// ---------------------------------------------------------------------------
// Q8_0 (32-element blocks; four blocks per warp iteration)
// ---------------------------------------------------------------------------
template <int NMG, int EPI>
__global__ void __launch_bounds__(256) k_qmv_q80(const uint8_t* __restrict__ W, int nblk,
                                                 int64_t rows, const uint4* __restrict__ xfrag,
                                                 const uint32_t* __restrict__ /*unused*/,
                                                 const float* __restrict__ xscale, int B,
                                                 float* __restrict__ y) {
  constexpr int U = 4;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2;
  const uint8_t* tile = W + (int64_t)blockIdx.x * nblk * 544;
  const int K32 = nblk;
  float tg[NMG], tg8[NMG];
#pragma unroll
  for (int i = 0; i < NMG; i++) tg[i] = tg8[i] = 0.f;
  bool waited = false;
  for (int b0 = warp * U; b0 < nblk; b0 += QMV_WARPS * U) {
    uint4 q[U];
    uint32_t dp[U];
#pragma unroll
    for (int u = 0; u < U; u++) {
      if (b0 + u < nblk) {
        const uint8_t* tb = tile + (int64_t)(b0 + u) * 544;
        q[u] = ldg_nc_v4(tb + lane * 16);
        dp[u] = *(const uint32_t*)(tb + 512 + 4 * g);
      } else {
        q[u] = make_uint4(0x80808080u, 0x80808080u, 0x80808080u, 0x80808080u);
        dp[u] = 0;
      }
    }
    if (!waited) {
      pdl_wait();
      waited = true;
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int bb = b0 + u < nblk ? b0 + u : nblk - 1;
      float C[NMG][4];
#pragma unroll
      for (int mg = 0; mg < NMG; mg++) C[mg][0] = C[mg][1] = C[mg][2] = C[mg][3] = 0.f;
      uint4 xf[NMG];
#pragma unroll
      for (int mg = 0; mg < NMG; mg++) xf[mg] = xfrag[((int64_t)mg * K32 + bb) * 32 + lane];
#pragma unroll
      for (int kt = 0; kt < 2; kt++) {
        const uint32_t wg = (kt ? q[u].z : q[u].x) ^ 0x80808080u;
        const uint32_t wg8 = (kt ? q[u].w : q[u].y) ^ 0x80808080u;
        const uint32_t a0 = hsub2_u32(prmt(wg, 0x64646464u, 0x5140u), 0x64806480u);
        const uint32_t a1 = hsub2_u32(prmt(wg8, 0x64646464u, 0x5140u), 0x64806480u);
        const uint32_t a2 = hsub2_u32(prmt(wg, 0x64646464u, 0x5342u), 0x64806480u);
        const uint32_t a3 = hsub2_u32(prmt(wg8, 0x64646464u, 0x5342u), 0x64806480u);
#pragma unroll
        for (int mg = 0; mg < NMG; mg++)
          mma16816(C[mg], a0, a1, a2, a3, kt ? xf[mg].z : xf[mg].x, kt ? xf[mg].w : xf[mg].y);
      }
      const float d0 = h2f_lo(dp[u]), d1 = h2f_hi(dp[u]);
#pragma unroll
      for (int mg = 0; mg < NMG; mg++) {
        tg[mg] += d0 * (C[mg][0] + C[mg][1]);
        tg8[mg] += d1 * (C[mg][2] + C[mg][3]);
      }
    }
  }
  if (!waited) pdl_wait();
  pdl_launch();
  qmv_epilogue<NMG, EPI>(tg, tg8, xscale, B, rows, y);
}

template <typename Kern>
int launch_k(Kern kern, cudaStream_t s, dim3 grid, dim3 block, size_t smem, bool pdl,
             const uint8_t* W, int nblk, int64_t rows, const uint4* xfrag, const uint32_t* xsfrag,
             const float* xscale, int B, float* y) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  SI_CUDA(cudaLaunchKernelEx(&cfg, kern, W, nblk, rows, xfrag, xsfrag, xscale, B, y));
  return SI_OK;
}

template <int NMG, int EPI>
int qmv_dispatch_qt(cudaStream_t s, const si_weight* w, const uint4* xfrag,
                    const uint32_t* xsfrag, const float* xscale, int B, float* y, bool pdl) {
  dim3 grid((unsigned)w->tiles), block(256);
  const uint8_t* W = (const uint8_t*)w->dev;
  switch (w->qtype) {
    case SI_Q4_K:
      return launch_k(k_qmv_q4k<NMG, EPI>, s, grid, block, 0, pdl, W, (int)w->nblk, w->rows, xfrag,
                      xsfrag, xscale, B, y);
    case SI_Q6_K:
      return launch_k(k_qmv_q6k<NMG, EPI>, s, grid, block, 0, pdl, W, (int)w->nblk, w->rows, xfrag,
                      xsfrag, xscale, B, y);
    case SI_Q8_0:
      return launch_k(k_qmv_q80<NMG, EPI>, s, grid, block, 0, pdl, W, (int)w->nblk, w->rows, xfrag,
                      xsfrag, xscale, B, y);
    default:
      SI_FAIL(SI_ERR_UNSUPPORTED, "qmatvec: unsupported quant type %d", w->qtype);
  }
}

template <int EPI>
int qmv_dispatch_nmg(cudaStream_t s, const si_weight* w, const uint4* xfrag,
                     const uint32_t* xsfrag, const float* xscale, int B, float* y, bool pdl) {
  switch ((B + 3) / 4) {
    case 1: return qmv_dispatch_qt<1, EPI>(s, w, xfrag, xsfrag, xscale, B, y, pdl);
    case 2: return qmv_dispatch_qt<2, EPI>(s, w, xfrag, xsfrag, xscale, B, y, pdl);
    case 3: return qmv_dispatch_qt<3, EPI>(s, w, xfrag, xsfrag, xscale, B, y, pdl);
    case 4: return qmv_dispatch_qt<4, EPI>(s, w, xfrag, xsfrag, xscale, B, y, pdl);
    default: SI_FAIL(SI_ERR_INVALID, "qmatvec: batch %d outside 1..16", B);
  }
}

}  // namespace

int prep_smem_bytes(int K) { return K * 4; }

int launch_prep(cudaStream_t s, const float* x, const float* x2, const float* norm_w, float eps,
                int mode, int K, int B, float* xout, uint4* xfrag, uint32_t* xsfrag,
                float* xscale, bool pdl) {
  if (K <= 0 || (K & 31)) SI_FAIL(SI_ERR_INVALID, "prep: K=%d must be a positive multiple of 32", K);
  if (K > SI_MAX_K) SI_FAIL(SI_ERR_INVALID, "prep: K=%d above the supported maximum %d", K, SI_MAX_K);
  const int nmg = (B + 3) / 4;
  size_t smem = (size_t)K * 4;
  static uint64_t attr_set = 0;  // one bit per device
  int dev = 0;
  SI_CUDA(cudaGetDevice(&dev));
  if (dev < 64 && !(attr_set & (1ull << dev))) {
    SI_CUDA(cudaFuncSetAttribute(k_prep, cudaFuncAttributeMaxDynamicSharedMemorySize, SI_MAX_K * 4));
    attr_set |= 1ull << dev;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nmg * 4);
  cfg.blockDim = dim3(512);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  SI_CUDA(cudaLaunchKernelEx(&cfg, k_prep, x, x2, norm_w, eps, mode, K, B, xout, xfrag, xsfrag,
                             xscale));
  return SI_OK;
}

int launch_qmv(cudaStream_t s, const si_weight* w, const uint4* xfrag, const uint32_t* xsfrag,
               const float* xscale, int B, float* y, int epi, bool pdl) {
  if (epi == SI_EPI_ADD) return qmv_dispatch_nmg<SI_EPI_ADD>(s, w, xfrag, xsfrag, xscale, B, y, pdl);
  return qmv_dispatch_nmg<SI_EPI_STORE>(s, w, xfrag, xsfrag, xscale, B, y, pdl);
}

}  // namespace si
