// Prefill GEMM on the 5th-generation tensor cores: Y[M][N] = X[M][K] W[N][K]^T
// for a K-quant weight W and bf16 activations X -- the batched form of the
// quantised MatVecMul that prefill needs (TensorOps.MatMul semantics,
// src/SharpInfer.Core/Tensors/TensorOps.cs:79-112, over the weights
// DequantizeTensor produces, Quantization.cs:415-469).
//
// Pipeline (one call):
//  1. W to f16.  Q4_K with M <= 896: inside the GEMM (k_gemm_q4k), eight
//     warps dequantise each 64-column step into the shared-memory B tile in
//     f16x2 arithmetic, about 3 instructions per 2 weights, which hides under
//     the tensor cores while each weight is dequantised by few row blocks.
//     Otherwise (larger M, Q6_K, Q8_0) a pre-pass (k_dequant_f16) writes f16
//     [N][K] to a context scratch buffer: element = the reference's f32 value
//     d*sc*q - dmin*m, rounded to f16 once.  si_qgemm_cache_weight keeps that
//     copy for later calls.
//  2. k_bf16_rows_to_f16: X -> f16, each row scaled by a power of two that
//     puts its largest |x| in [2^14, 2^15) (undone in the epilogue), so the
//     whole bf16 range converts without overflow; kind::f16 needs A and B of
//     one type, and f16 keeps 3 more mantissa bits of W than bf16.
//  3. k_gemm_tc: 128 x 256 output tile per CTA, K in steps of 64.  Warp 0
//     issues TMA loads (128B-swizzled, 4-stage mbarrier ring), warp 1 issues
//     tcgen05.mma (kind::f16, f32 accumulator in TMEM, 4 MMAs of K = 16 per
//     stage) and tcgen05.commit to free stages, warps 2-5 read the
//     accumulator back with tcgen05.ld and store Y.
// Accuracy: W's f16 rounding (2^-12 relative; in the fused kernel also the
// f16 rounding of d*sc and dmin*m and of the HFMA2), ~1e-4 relative L2 on Y.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "quantfmt.cuh"
#include "tcgen05.cuh"

namespace si {
namespace {

constexpr int GM = 128, GK = 64, GST = 4;
constexpr int A_BYTES = GM * GK * 2;  // 16 KB
template <int BN>
struct GemmCfg {
  static constexpr int B_BYTES = BN * GK * 2;  // 32 KB at BN = 256
  static constexpr int SMEM = GST * (A_BYTES + B_BYTES) + 1024 + 256;
  // kind::f16 instruction descriptor: D f32, A and B f16, both K-major, N = BN, M = GM.
  static constexpr uint32_t IDESC = (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(GM >> 4) << 24);
};

// f16 of one (row, block) in the reference's f32 arithmetic.
__global__ void k_dequant_f16(int qt, const uint8_t* __restrict__ W, int64_t rows, int64_t nblk,
                              __half* __restrict__ out) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= rows * nblk) return;
  const int64_t r = idx / nblk, b = idx % nblk;
  const int64_t T = r >> 4;
  const int ri = (int)(r & 15);
  const int be = qt == SI_Q8_0 ? 32 : 256;
  __half* o = out + r * nblk * be + b * be;
  if (qt == SI_Q4_K) {
    const uint32_t* tbw = (const uint32_t*)(W + (T * nblk + b) * 2304);
    const uint8_t* hdr = (const uint8_t*)(tbw + 4 * ri);
    const float d = h2f(hdr[0] | (hdr[1] << 8)), dmin = h2f(hdr[2] | (hdr[3] << 8));
    const uint8_t* q = hdr + 4;
    for (int j = 0; j < 8; j++) {  // GetScaleMinK4 (Quantization.cs:302-314)
      uint32_t sc, mn;
      if (j < 4) {
        sc = q[j] & 63;
        mn = q[j + 4] & 63;
      } else {
        sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        mn = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
      }
      const float d1 = __fmul_rn(d, (float)sc), m1f = __fmul_rn(dmin, (float)mn);
      for (int l0 = 0; l0 < 32; l0 += 8) {
        __align__(16) __half v[8];
#pragma unroll
        for (int l = 0; l < 8; l++)
          v[l] = __float2half_rn(__fsub_rn(__fmul_rn(d1, (float)dev_q4k_code(tbw, ri, 32 * j + l0 + l)), m1f));
        *(uint4*)(o + 32 * j + l0) = *(const uint4*)v;
      }
    }
  } else if (qt == SI_Q6_K) {
    const uint32_t* tbw = (const uint32_t*)(W + (T * nblk + b) * 3360);
    const int8_t* scales = (const int8_t*)(tbw + 768) + 16 * ri;
    const uint32_t dw = tbw[832 + (ri & 7)];
    const float d = h2f((ri >> 3) ? (dw >> 16) : (dw & 0xFFFF));
    for (int e0 = 0; e0 < 256; e0 += 8) {
      __align__(16) __half v[8];
#pragma unroll
      for (int l = 0; l < 8; l++) {
        const int e = e0 + l;
        const float ds = __fmul_rn(d, (float)scales[e >> 4]);
        v[l] = __float2half_rn(__fmul_rn(ds, (float)((int)dev_q6k_code(tbw, ri, e) - 32)));
      }
      *(uint4*)(o + e0) = *(const uint4*)v;
    }
  } else {
    const uint32_t* tbw = (const uint32_t*)(W + (T * nblk + b) * 544);
    const uint32_t dw = tbw[128 + (ri & 7)];
    const float d = h2f((ri >> 3) ? (dw >> 16) : (dw & 0xFFFF));
    for (int e0 = 0; e0 < 32; e0 += 8) {
      __align__(16) __half v[8];
#pragma unroll
      for (int l = 0; l < 8; l++) v[l] = __float2half_rn(__fmul_rn((float)dev_q80_code(tbw, ri, e0 + l), d));
      *(uint4*)(o + e0) = *(const uint4*)v;
    }
  }
}

// Q4_K: one warp per 16-row tile-block, reading the fragment-ordered words
// directly (lane (g, t), word i of chunk c = k-tile 4c + i, rows g and g+8).
__global__ void __launch_bounds__(256) k_dequant_q4k_f16(const uint8_t* __restrict__ W, int64_t rows, int64_t nblk,
                                                         int64_t ntb, __half* __restrict__ out) {
  const int64_t tb = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (tb >= ntb) return;
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int64_t T = tb / nblk, b = tb % nblk;
  const uint32_t* tbw = (const uint32_t*)(W + tb * 2304);
  const int64_t K = nblk * 256;
  float d1[2][8], m1[2][8];
#pragma unroll
  for (int h = 0; h < 2; h++) {  // rows g, g+8: GetScaleMinK4 (Quantization.cs:302-314)
    const uint4 hd = *(const uint4*)(tbw + 4 * (g + 8 * h));
    const float d = h2f(hd.x & 0xFFFF), dmin = h2f(hd.x >> 16);
    const uint32_t qw[3] = {hd.y, hd.z, hd.w};
#pragma unroll
    for (int j = 0; j < 8; j++) {
      auto qb = [&](int k) { return (qw[k >> 2] >> (8 * (k & 3))) & 0xFF; };
      uint32_t sc, mn;
      if (j < 4) {
        sc = qb(j) & 63;
        mn = qb(j + 4) & 63;
      } else {
        sc = (qb(j + 4) & 0xF) | ((qb(j - 4) >> 6) << 4);
        mn = (qb(j + 4) >> 4) | ((qb(j) >> 6) << 4);
      }
      d1[h][j] = __fmul_rn(d, (float)sc);
      m1[h][j] = __fmul_rn(dmin, (float)mn);
    }
  }
#pragma unroll
  for (int c = 0; c < 4; c++) {
    const uint4 q = *(const uint4*)(tbw + 64 + c * 128 + lane * 4);
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const uint32_t w = i == 0 ? q.x : i == 1 ? q.y : i == 2 ? q.z : q.w;
      const int kt = 4 * c + i, s = kt >> 1;
      const int64_t col = b * 256 + 16 * kt + 2 * t;
#pragma unroll
      for (int h = 0; h < 2; h++) {
        const int64_t r = T * 16 + g + 8 * h;
        if (r >= rows) continue;
        const int sh = 4 * h;
        auto v = [&](int bit) {
          return __float2half_rn(__fsub_rn(__fmul_rn(d1[h][s], (float)((w >> (bit + sh)) & 0xF)), m1[h][s]));
        };
        __half* o = out + r * K + col;
        *(__half2*)o = __halves2half2(v(0), v(16));
        *(__half2*)(o + 8) = __halves2half2(v(8), v(24));
      }
    }
  }
}

// Row m of X -> f16 scaled by 2^e_m, with e_m chosen so that the row's
// largest |x| lands in [2^14, 2^15); rs[m] = 2^-e_m undoes the scale in the
// GEMM epilogue.  Every product and f32 sum then carries the factor 2^e_m
// exactly, so y is what unscaled f16 arithmetic would give -- but no bf16
// value overflows f16 (|x| up to 3.4e38) and none below f16's normal range
// (6.1e-5) loses bits unless it lies more than 2^28 under its row's maximum,
// where its share of the row's products is below 2^-28 of the largest.
__global__ void __launch_bounds__(256) k_bf16_rows_to_f16(const uint16_t* __restrict__ x, __half* __restrict__ y,
                                                          float* __restrict__ rs, int K) {
  __shared__ uint32_t red[8];
  const int m = blockIdx.x, tid = threadIdx.x;
  const uint4* xr = (const uint4*)(x + (int64_t)m * K);
  uint4* yr = (uint4*)(y + (int64_t)m * K);
  const int n8 = K / 8;  // K is a multiple of 64
  pdl_launch();
  pdl_wait();
  // the largest magnitude from the bits: |x| orders like its bits with the sign cleared
  uint32_t mb = 0;
  for (int i = tid; i < n8; i += 256) {
    const uint4 v = xr[i];
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int k = 0; k < 4; k++) mb = max(mb, max(w[k] & 0x7FFFu, (w[k] >> 16) & 0x7FFFu));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mb = max(mb, __shfl_xor_sync(0xFFFFFFFFu, mb, o));
  if ((tid & 31) == 0) red[tid >> 5] = mb;
  __syncthreads();
  mb = 0;
#pragma unroll
  for (int i = 0; i < 8; i++) mb = max(mb, red[i]);
  int e = 0;
  if (mb != 0 && mb < 0x7F80u) {  // finite, non-zero maximum
    const int E = (int)(mb >> 7) - 127;  // its binary exponent (bf16 subnormals count as 2^-127)
    e = 14 - E;
    e = e < -100 ? -100 : (e > 100 ? 100 : e);
  }
  const float sc = ldexpf(1.0f, e);
  if (tid == 0) rs[m] = ldexpf(1.0f, -e);
  for (int i = tid; i < n8; i += 256) {
    const uint4 v = xr[i];
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const __half lo = __float2half_rn(__uint_as_float(w[k] << 16) * sc);
      const __half hi = __float2half_rn(__uint_as_float(w[k] & 0xFFFF0000u) * sc);
      o[k] = (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
    }
    yr[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

template <int GN>
__global__ void __launch_bounds__(192, 1) k_gemm_tc(const __grid_constant__ CUtensorMap tmA,
                                                    const __grid_constant__ CUtensorMap tmB, float* __restrict__ Y,
                                                    const float* __restrict__ rs, int M, int N, int K, int acc,
                                                    int* err) {
  constexpr int B_BYTES = GemmCfg<GN>::B_BYTES;
  constexpr uint32_t IDESC = GemmCfg<GN>::IDESC;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t sA = base, sB = base + GST * A_BYTES, bars = sB + GST * B_BYTES;
  const uint32_t done = bars + 64, tslot = bars + 72;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * GM, n0 = blockIdx.x * GN, nk = K / GK;
  if (threadIdx.x == 0) {
    for (int s = 0; s < GST; s++) {
      mbar_init(bars + 8 * s, 1);       // full: TMA bytes landed
      mbar_init(bars + 32 + 8 * s, 1);  // empty: MMAs reading the stage are done
    }
    mbar_init(done, 1);
    mbar_fence_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tslot), "r"(GN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = lds_u32(tslot);
  pdl_launch();  // dependents may start their independent prologue now
  pdl_wait();    // A and B are written by the preceding conversion kernels

  bool ok = true;
  if (warp == 0) {
    if (lane == 0) {  // TMA producer
      for (int kt = 0; kt < nk && ok; kt++) {
        const int s = kt % GST;
        if (kt >= GST && !mbar_wait_bounded(bars + 32 + 8 * s, (uint32_t)((kt / GST - 1) & 1))) ok = false;
        mbar_arrive_expect_tx(bars + 8 * s, A_BYTES + B_BYTES);
        tma_load_2d(sA + s * A_BYTES, &tmA, kt * GK, m0, bars + 8 * s);
        tma_load_2d(sB + s * B_BYTES, &tmB, kt * GK, n0, bars + 8 * s);
      }
      if (!ok) atomicOr(err, SI_DEVERR_WAIT_TIMEOUT);
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      for (int kt = 0; kt < nk; kt++) {
        const int s = kt % GST;
        if (ok && !mbar_wait_bounded(bars + 8 * s, (uint32_t)((kt / GST) & 1))) ok = false;
        tc_fence_after();
        if (ok) {
          const uint64_t da = sdesc_k128(sA + s * A_BYTES), db = sdesc_k128(sB + s * B_BYTES);
#pragma unroll
          for (int kk = 0; kk < GK / 16; kk++)  // +32 B along K per MMA inside the swizzle atom
            umma_f16(tmem, da + 2 * kk, db + 2 * kk, IDESC, (kt | kk) != 0);
        }
        umma_commit(bars + 32 + 8 * s);
      }
      umma_commit(done);
      if (!ok) atomicOr(err, SI_DEVERR_WAIT_TIMEOUT);
    }
  } else {  // epilogue: TMEM lanes 32 (warp % 4) .. +31 = tile rows
    if (!mbar_wait_bounded(done, 0)) {
      ok = false;
      if (lane == 0) atomicOr(err, SI_DEVERR_WAIT_TIMEOUT);
    }
    tc_fence_after();
    const int q = warp & 3;
    const int row = m0 + 32 * q + lane;
    float* yr = Y + (int64_t)row * N;
    const float rsc = row < M ? rs[row] : 0.f;  // the row's 2^-e
    for (int c0 = 0; c0 < GN; c0 += 32) {
      uint32_t r[32];
      tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)c0, r);
      if (!ok || row >= M) continue;
      const int col0 = n0 + c0;
      if (col0 + 32 <= N && (N & 3) == 0) {
#pragma unroll
        for (int j = 0; j < 32; j += 4)
        {
          float4 v = make_float4(__uint_as_float(r[j]) * rsc, __uint_as_float(r[j + 1]) * rsc,
                                 __uint_as_float(r[j + 2]) * rsc, __uint_as_float(r[j + 3]) * rsc);
          if (acc) {
            const float4 o = *(const float4*)(yr + col0 + j);
            v = make_float4(o.x + v.x, o.y + v.y, o.z + v.z, o.w + v.w);
          }
          *(float4*)(yr + col0 + j) = v;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; j++)
          if (col0 + j < N) yr[col0 + j] = (acc ? yr[col0 + j] : 0.f) + __uint_as_float(r[j]) * rsc;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(GN) : "memory");
  }
}

// Q4_K GEMM with the weight dequantised in shared memory (no f16 copy of W):
// the same tile and warp plan as k_gemm_tc, except that B is produced by
// eight dequantising warps (2-9) instead of TMA.  A 64-column K step is one
// 512-byte nibble chunk of a tile-block (4 k-tiles), so for each of its
// BN / 128 row tiles a lane loads one 16-byte word group (rows g and g+8,
// k = 2t, 2t+1, 2t+8, 2t+9 of the chunk's 4 k-tiles) and writes 16 f16
// pairs into the 128-byte-swizzled K-major B tile (conflict free: the 16-byte
// chunk index is XORed with g).  Values are computed in f16x2:
// (1024 + q) from the nibble bits (the device layout's exact f16 pairs),
// minus 1024, times d*sc plus -dmin*m (both rounded to f16 once per
// sub-block) -- one HFMA2 per pair.  The superblock header and the next
// chunk are loaded one step ahead.  After the main loop warps 2-5 drain the
// accumulator as in k_gemm_tc.  All waits are bounded; after one gives up, a
// thread waits no more.
__device__ __forceinline__ __half2 u2h2(uint32_t v) { return *(__half2*)&v; }
__device__ __forceinline__ uint32_t h22u(__half2 v) { return *(uint32_t*)&v; }
__device__ __forceinline__ uint32_t lop_and_or(uint32_t a, uint32_t m, uint32_t o) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(m), "r"(o));  // (a & m) | o
  return r;
}

template <int GN>
__global__ void __launch_bounds__(320, 1) k_gemm_q4k(const __grid_constant__ CUtensorMap tmA, const uint8_t* __restrict__ W,
                                                     int tiles, float* __restrict__ Y, const float* __restrict__ rs, int M,
                                                     int N, int K, int acc, int* err) {
  constexpr int B_BYTES = GemmCfg<GN>::B_BYTES;
  constexpr uint32_t IDESC = GemmCfg<GN>::IDESC;
  constexpr int RT = GN / 128;  // row tiles per dequantising warp
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t sA = base, sB = base + GST * A_BYTES, bars = sB + GST * B_BYTES;
  // a_full[GST] b_full[GST] empty[GST] done, TMEM slot
  const uint32_t a_full = bars, b_full = bars + 8 * GST, empty = bars + 16 * GST, done = bars + 24 * GST,
                 tslot = done + 8;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * GM, n0 = blockIdx.x * GN, nk = K / GK, nblk = K / 256;
  if (threadIdx.x == 0) {
    for (int s = 0; s < GST; s++) {
      mbar_init(a_full + 8 * s, 1);
      mbar_init(b_full + 8 * s, 256);
      mbar_init(empty + 8 * s, 1);
    }
    mbar_init(done, 1);
    mbar_fence_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tslot), "r"(GN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = lds_u32(tslot);
  pdl_launch();
  pdl_wait();  // A is written by the preceding conversion kernel

  bool ok = true;
  if (warp == 0) {
    if (lane == 0) {  // TMA producer of A
      for (int kt = 0; kt < nk && ok; kt++) {
        const int s = kt % GST;
        if (kt >= GST && !mbar_wait_bounded(empty + 8 * s, (uint32_t)((kt / GST - 1) & 1))) ok = false;
        mbar_arrive_expect_tx(a_full + 8 * s, A_BYTES);
        tma_load_2d(sA + s * A_BYTES, &tmA, kt * GK, m0, a_full + 8 * s);
      }
      if (!ok) atomicOr(err, SI_DEVERR_WAIT_TIMEOUT);
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      for (int kt = 0; kt < nk; kt++) {
        const int s = kt % GST;
        if (ok && !mbar_wait_bounded(a_full + 8 * s, (uint32_t)((kt / GST) & 1))) ok = false;
        if (ok && !mbar_wait_bounded(b_full + 8 * s, (uint32_t)((kt / GST) & 1))) ok = false;
        tc_fence_after();
        if (ok) {
          const uint64_t da = sdesc_k128(sA + s * A_BYTES), db = sdesc_k128(sB + s * B_BYTES);
#pragma unroll
          for (int kk = 0; kk < GK / 16; kk++) umma_f16(tmem, da + 2 * kk, db + 2 * kk, IDESC, (kt | kk) != 0);
        }
        umma_commit(empty + 8 * s);
      }
      umma_commit(done);
      if (!ok) atomicOr(err, SI_DEVERR_WAIT_TIMEOUT);
    }
  } else {
    {  // B producers: dequantising warp dw takes row tiles dw and dw + 8 of the CTA's GN rows
      const int dw = warp - 2, g = lane >> 2, t = lane & 3;
      const uint8_t* tb[RT];
      bool have[RT];
#pragma unroll
      for (int rt = 0; rt < RT; rt++) {
        const int Tg = n0 / 16 + dw + 8 * rt;
        have[rt] = Tg < tiles;
        tb[rt] = W + (int64_t)(have[rt] ? Tg : 0) * nblk * 2304;
      }
      uint4 qc[RT], hc[RT][2];  // this step's nibble words; this superblock's headers (rows g, g+8)
#pragma unroll
      for (int rt = 0; rt < RT; rt++) {
        qc[rt] = __ldg((const uint4*)(tb[rt] + 256 + 16 * lane));
        hc[rt][0] = __ldg((const uint4*)(tb[rt] + 16 * g));
        hc[rt][1] = __ldg((const uint4*)(tb[rt] + 16 * (g + 8)));
      }
      uint32_t ds[RT][2][8], nm[RT][2][8];  // (d sc, d sc) and (-dmin m, -dmin m) per sub-block; row g+8: d sc / 16
      for (int sb = 0; sb < nblk; sb++) {
#pragma unroll
        for (int rt = 0; rt < RT; rt++)
#pragma unroll
          for (int h = 0; h < 2; h++) {  // GetScaleMinK4 (Quantization.cs:302-314)
            const uint4 hd = hc[rt][h];
            const float d = h2f(hd.x & 0xFFFF), dmin = h2f(hd.x >> 16);
            const uint32_t qw[3] = {hd.y, hd.z, hd.w};
#pragma unroll
            for (int j = 0; j < 8; j++) {
              auto qb = [&](int k) { return (qw[k >> 2] >> (8 * (k & 3))) & 0xFF; };
              uint32_t sc, mn;
              if (j < 4) {
                sc = qb(j) & 63;
                mn = qb(j + 4) & 63;
              } else {
                sc = (qb(j + 4) & 0xF) | ((qb(j - 4) >> 6) << 4);
                mn = (qb(j + 4) >> 4) | ((qb(j) >> 6) << 4);
              }
              const float dsc = __fmul_rn(d, (float)sc) * (h ? 0.0625f : 1.0f);
              const float ndm = -__fmul_rn(dmin, (float)mn);
              ds[rt][h][j] = h22u(__float2half2_rn(dsc));
              nm[rt][h][j] = h22u(__float2half2_rn(ndm));
            }
          }
#pragma unroll
        for (int c = 0; c < 4; c++) {  // the superblock's four 64-column steps
          const int kt = 4 * sb + c, s = kt % GST, kn = kt + 1;
          uint4 qn[RT], hn[RT][2];  // one step ahead
          if (kn < nk) {
#pragma unroll
            for (int rt = 0; rt < RT; rt++) {
              const uint8_t* tbn = tb[rt] + (int64_t)(kn >> 2) * 2304;
              qn[rt] = __ldg((const uint4*)(tbn + 256 + 512 * (kn & 3) + 16 * lane));
              if (c == 3) {
                hn[rt][0] = __ldg((const uint4*)(tbn + 16 * g));
                hn[rt][1] = __ldg((const uint4*)(tbn + 16 * (g + 8)));
              }
            }
          }
          if (ok && kt >= GST && !mbar_wait_bounded(empty + 8 * s, (uint32_t)((kt / GST - 1) & 1))) ok = false;
          const uint32_t bst = sB + s * B_BYTES;
          const __half2 k1024 = u2h2(0x64006400u);
#pragma unroll
          for (int rt = 0; rt < RT; rt++) {
            if (!have[rt]) continue;  // rows past the weight: their output columns are not stored
            const uint32_t row0 = bst + (uint32_t)(16 * (dw + 8 * rt) + g) * 128u + 4u * t;  // row g; g + 8 at +1024
            const uint32_t q4[4] = {qc[rt].x, qc[rt].y, qc[rt].z, qc[rt].w};
#pragma unroll
            for (int i = 0; i < 4; i++) {  // k-tile 4c + i: groups of 8 columns 2i and 2i + 1
              const int j = 2 * c + (i >> 1);  // sub-block
              const uint32_t w = q4[i], w8 = w >> 8;
              const __half2 dg = u2h2(ds[rt][0][j]), mg = u2h2(nm[rt][0][j]);
              const __half2 d8 = u2h2(ds[rt][1][j]), m8 = u2h2(nm[rt][1][j]);
              const uint32_t a0 = h22u(__hfma2(__hsub2(u2h2(lop_and_or(w, 0x000F000Fu, 0x64006400u)), k1024), dg, mg));
              const uint32_t a1 = h22u(__hfma2(__hsub2(u2h2(lop_and_or(w8, 0x000F000Fu, 0x64006400u)), k1024), dg, mg));
              const uint32_t b0 = h22u(__hfma2(__hsub2(u2h2(lop_and_or(w, 0x00F000F0u, 0x64006400u)), k1024), d8, m8));
              const uint32_t b1 = h22u(__hfma2(__hsub2(u2h2(lop_and_or(w8, 0x00F000F0u, 0x64006400u)), k1024), d8, m8));
              const uint32_t c0 = (uint32_t)(((2 * i) ^ g) << 4), c1 = (uint32_t)(((2 * i + 1) ^ g) << 4);
              asm volatile("st.shared.u32 [%0], %1;" ::"r"(row0 + c0), "r"(a0) : "memory");
              asm volatile("st.shared.u32 [%0], %1;" ::"r"(row0 + c1), "r"(a1) : "memory");
              asm volatile("st.shared.u32 [%0], %1;" ::"r"(row0 + 1024u + c0), "r"(b0) : "memory");
              asm volatile("st.shared.u32 [%0], %1;" ::"r"(row0 + 1024u + c1), "r"(b1) : "memory");
            }
          }
          fence_proxy_async_smem();
          mbar_arrive(b_full + 8 * s);
          if (kn < nk) {
#pragma unroll
            for (int rt = 0; rt < RT; rt++) {
              qc[rt] = qn[rt];
              if (c == 3) {
                hc[rt][0] = hn[rt][0];
                hc[rt][1] = hn[rt][1];
              }
            }
          }
        }
      }
    }
    if (warp < 6) {  // epilogue: TMEM lanes 32 (warp % 4) .. +31 = tile rows
      if (ok && !mbar_wait_bounded(done, 0)) ok = false;
      if (!ok && lane == 0) atomicOr(err, SI_DEVERR_WAIT_TIMEOUT);
      tc_fence_after();
      const int q = warp & 3;
      const int row = m0 + 32 * q + lane;
      float* yr = Y + (int64_t)row * N;
      const float rsc = row < M ? rs[row] : 0.f;  // the row's 2^-e
      for (int c0 = 0; c0 < GN; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)c0, r);
        if (!ok || row >= M) continue;
        const int col0 = n0 + c0;
        if (col0 + 32 <= N && (N & 3) == 0) {
#pragma unroll
          for (int j = 0; j < 32; j += 4)
          {
            float4 v = make_float4(__uint_as_float(r[j]) * rsc, __uint_as_float(r[j + 1]) * rsc,
                                   __uint_as_float(r[j + 2]) * rsc, __uint_as_float(r[j + 3]) * rsc);
            if (acc) {
              const float4 o = *(const float4*)(yr + col0 + j);
              v = make_float4(o.x + v.x, o.y + v.y, o.z + v.z, o.w + v.w);
            }
            *(float4*)(yr + col0 + j) = v;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; j++)
            if (col0 + j < N) yr[col0 + j] = (acc ? yr[col0 + j] : 0.f) + __uint_as_float(r[j]) * rsc;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(GN) : "memory");
  }
}

// 2D f16 tensor [rows][cols] (row-major), box [box_rows][64], 128-byte swizzle.
int make_tmap(CUtensorMap* tm, const void* ptr, int64_t rows, int64_t cols, int box_rows) {
  auto fn = encode_fn();
  if (!fn) SI_FAIL(SI_ERR_CUDA, "qgemm: cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  const cuuint32_t box[2] = {(cuuint32_t)GK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) SI_FAIL(SI_ERR_CUDA, "qgemm: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return SI_OK;
}

}  // namespace

// f16 copy of W (rows x cols) at dst on the context stream.
int dequant_f16(si_ctx* c, const si_weight* w, __half* dst) {
  const int64_t N = w->rows;
  if (raw_layout(w->qtype)) return launch_dequant_raw_f16(c->stream, w, dst);
  if (w->qtype == SI_Q4_K) {
    const int64_t ntb = w->tiles * w->nblk;
    k_dequant_q4k_f16<<<(unsigned)((ntb + 7) / 8), 256, 0, c->stream>>>((const uint8_t*)w->dev, N, w->nblk, ntb, dst);
  } else {
    const int64_t nb = N * w->nblk;
    k_dequant_f16<<<(unsigned)((nb + 127) / 128), 128, 0, c->stream>>>(w->qtype, (const uint8_t*)w->dev, N, w->nblk,
                                                                        dst);
  }
  SI_CUDA(cudaGetLastError());
  return SI_OK;
}

int launch_qgemm(si_ctx* c, const si_weight* w, const uint16_t* x, float* y, int M) {
  const int64_t K = w->cols;
  if (K % GK) SI_FAIL(SI_ERR_UNSUPPORTED, "qgemm: cols %lld not a multiple of %d", (long long)K, GK);
  const size_t xbytes = ((size_t)M * K * 2 + 255) & ~(size_t)255;
  SI_TRY(ensure(c->stage[1], xbytes + (size_t)M * 4));
  __half* xf = (__half*)c->stage[1].ptr;
  float* rs = (float*)((uint8_t*)c->stage[1].ptr + xbytes);  // per-row 2^-e of the conversion
  if (((uintptr_t)x & 15) != 0) SI_FAIL(SI_ERR_INVALID, "si_qgemm: x must be 16-byte aligned");
  k_bf16_rows_to_f16<<<(unsigned)M, 256, 0, c->stream>>>(x, xf, rs, (int)K);
  SI_CUDA(cudaGetLastError());
  return launch_qgemm_f16in(c, w, xf, rs, y, M, 0);
}

// y[m] (+)= rs[m] * (xf[m] . W) for f16 rows xf [M][cols] (16-byte aligned)
// already scaled by 2^e per row (rs[m] = 2^-e); accumulate != 0 adds to y.
int launch_qgemm_f16in(si_ctx* c, const si_weight* w, const __half* xf, const float* rs, float* y, int M,
                       int accumulate) {
  const int64_t N = w->rows, K = w->cols;
  if (K % GK) SI_FAIL(SI_ERR_UNSUPPORTED, "qgemm: cols %lld not a multiple of %d", (long long)K, GK);
  __half* wf = (__half*)w->f16;
  // Q4_K without a cached copy: dequantised in shared memory while the row
  // blocks of X are few (each one dequantises W again; measured on the 8B
  // shapes the fused kernel wins at M = 512 and loses at M = 2048 to the
  // pre-pass, crossing near M = 900).
  const bool fused = !wf && w->qtype == SI_Q4_K && (M + GM - 1) / GM <= 7;
  if (!wf && !fused) {  // no cached copy: dequantise into scratch for this call
    SI_TRY(ensure(c->stage[0], (size_t)N * K * 2));
    wf = (__half*)c->stage[0].ptr;
    SI_TRY(dequant_f16(c, w, wf));
  }
  // 256-wide tiles, or 128-wide when 256 would leave SMs idle
  const int64_t tiles256 = ((N + 255) / 256) * (((int64_t)M + GM - 1) / GM);
  const int GN = tiles256 < c->sm_count ? 128 : 256;
  CUtensorMap ta, tb;
  SI_TRY(make_tmap(&ta, xf, M, K, GM));
  if (fused) {
    static DeviceOnce fattr[2];
    const int fi = GN == 128 ? 0 : 1;
    const int fsmem = GN == 128 ? GemmCfg<128>::SMEM : GemmCfg<256>::SMEM;
    if (!fattr[fi].done(c->device)) {
      if (GN == 128) SI_CUDA(cudaFuncSetAttribute(k_gemm_q4k<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, fsmem));
      else SI_CUDA(cudaFuncSetAttribute(k_gemm_q4k<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, fsmem));
      fattr[fi].mark(c->device);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((N + GN - 1) / GN), (unsigned)((M + GM - 1) / GM));
    cfg.blockDim = dim3(320);
    cfg.dynamicSmemBytes = fsmem;
    cfg.stream = c->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const uint8_t* wd = (const uint8_t*)w->dev;
    if (GN == 128)
      SI_CUDA(cudaLaunchKernelEx(&cfg, k_gemm_q4k<128>, ta, wd, (int)w->tiles, y, rs, M, (int)N, (int)K, accumulate,
                                 c->dev_err));
    else
      SI_CUDA(cudaLaunchKernelEx(&cfg, k_gemm_q4k<256>, ta, wd, (int)w->tiles, y, rs, M, (int)N, (int)K, accumulate,
                                 c->dev_err));
    return SI_OK;
  }
  SI_TRY(make_tmap(&tb, wf, N, K, GN));
  static DeviceOnce attr_set[2];
  const int ai = GN == 128 ? 0 : 1;
  const int smem = GN == 128 ? GemmCfg<128>::SMEM : GemmCfg<256>::SMEM;
  if (!attr_set[ai].done(c->device)) {
    if (GN == 128) SI_CUDA(cudaFuncSetAttribute(k_gemm_tc<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    else SI_CUDA(cudaFuncSetAttribute(k_gemm_tc<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr_set[ai].mark(c->device);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((N + GN - 1) / GN), (unsigned)((M + GM - 1) / GM));
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = c->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (GN == 128)
    SI_CUDA(cudaLaunchKernelEx(&cfg, k_gemm_tc<128>, ta, tb, y, rs, M, (int)N, (int)K, accumulate, c->dev_err));
  else
    SI_CUDA(cudaLaunchKernelEx(&cfg, k_gemm_tc<256>, ta, tb, y, rs, M, (int)N, (int)K, accumulate, c->dev_err));
  return SI_OK;
}

}  // namespace si

using namespace si;

extern "C" SI_EXPORT int si_qgemm_cache_weight(si_ctx* c, si_weight* w) {
  clear_error();
  if (!c || !w) SI_FAIL(SI_ERR_INVALID, "si_qgemm_cache_weight: NULL argument");
  if (w->device != c->device) SI_FAIL(SI_ERR_INVALID, "si_qgemm_cache_weight: weight on device %d, context on %d",
                                      w->device, c->device);
  if (w->f16) return SI_OK;
  SI_TRY(bind_device(c));
  void* p = nullptr;
  const size_t bytes = (size_t)w->rows * w->cols * 2;
  const cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess)
    SI_FAIL(e == cudaErrorMemoryAllocation ? SI_ERR_OOM : SI_ERR_CUDA, "cudaMalloc(%zu) failed: %s", bytes,
            cudaGetErrorString(e));
  const int st = dequant_f16(c, w, (__half*)p);
  if (st != SI_OK || cudaStreamSynchronize(c->stream) != cudaSuccess) {
    cudaFree(p);
    return st != SI_OK ? st : SI_ERR_CUDA;
  }
  w->f16 = p;
  return SI_OK;
}

extern "C" SI_EXPORT int si_qgemm(si_ctx* c, const si_weight* w, const uint16_t* x_bf16, float* y, int M) {
  clear_error();
  if (!c || !w || !x_bf16 || !y) SI_FAIL(SI_ERR_INVALID, "si_qgemm: NULL argument");
  if (M < 1) SI_FAIL(SI_ERR_INVALID, "si_qgemm: M = %d", M);
  if (w->device != c->device) SI_FAIL(SI_ERR_INVALID, "si_qgemm: weight on device %d, context on %d", w->device, c->device);
  SI_TRY(bind_device(c));
  return launch_qgemm(c, w, x_bf16, y, M);
}
