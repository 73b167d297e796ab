// Fused dequantise + matvec for Q4_K / Q6_K / Q8_0 weights, batch 1..16.
//
// y[b][r] = sum_c W[r][c] x[b][c]  -- the quantised form of
// TensorOps.MatVecMul (src/SharpInfer.Core/Tensors/TensorOps.cs:63-72) with W
// decoded as in Quantization.cs (Q4_K :273-314, Q6_K :362-391, Q8_0 :106-114).
//
// The kernel is bound by HBM: every weight byte is read once.  To keep the
// instruction rate below the byte rate, the multiply-adds run on the tensor
// cores (mma.m16n8k16, f16 inputs, f32 accumulation):
//  * quant codes are small integers and exact in f16; for Q4_K a nibble
//    masked in place is the f16 subnormal q * 2^-24 (or 16q * 2^-24), and
//    one f16 multiply by the 6-bit sub-block scale gives q*sc*2^-24 exactly
//    (q*sc <= 945 fits the subnormal grid);
//  * activations are split into f16 hi + lo parts (x*2^e = hi + lo, ~22
//    significant bits, e chosen per 256-column unit) that occupy two MMA
//    columns, so the product keeps f32-level accuracy; batch b uses columns
//    2(b%4), 2(b%4)+1 of MMA group b/4;
//  * the Q4_K mins term dmin * sum_s m_s * X_s (X_s = sum of x over the 32
//    elements of sub-block s) is one more MMA per block.
// A row tile of 16 rows is one CTA of 8 warps; the warps split the K range
// in units of 256 columns and are reduced through shared memory at the end.
//
// Batch <= 4: each warp streams its units through its own shared-memory ring
// (cp.async.bulk on the TMA engine, one mbarrier per stage): the 16-row
// weight tile-block and the unit's prepared activations arrive together, so
// no load sits on the critical path of the MMAs.  Batch 5..16 reads the
// weights and activations straight from global memory.
#include "common.cuh"
#include "prepfmt.cuh"

namespace si {
namespace {

constexpr int QMV_WARPS = 8;
__device__ __forceinline__ float h2f_lo(uint32_t w) {
  return __half2float(__ushort_as_half((unsigned short)(w & 0xFFFF)));
}
__device__ __forceinline__ float h2f_hi(uint32_t w) {
  return __half2float(__ushort_as_half((unsigned short)(w >> 16)));
}

// ---------------------------------------------------------------------------
// Activation preparation.  One CTA per (256-column unit u, batch row b).
//   mode 0: v = x
//   mode 1: v = RmsNorm(x) * w   (TensorOps.cs:135-145); every CTA of a row
//           computes the row's sum of squares in the same order
//   mode 2: v = SiLU(x) * x2     (TensorOps.cs:191-195 then :169-185)
//   mode 3: v = attention output merged from split-KV partials: x is
//           o [B][K/128 heads][S][128] (unnormalised), x2 is (max, sum)
//           [B][heads][S][2], ldx = S.  For head h: M = max_s m_s,
//           w_s = exp(m_s - M), v = sum_s w_s o_s / sum_s w_s l_s -- the
//           softmax of Transformer.cs:99-129 over all positions, assembled
//           from the splits.
// x row b starts at x + b*ldx (x2 likewise; modes 0-2).  The unit's values are scaled by
// 2^e (max |v * 2^e| in [2^13, 2^14)), split into f16 hi/lo fragments for
// the lanes 8(b%4) .. 8(b%4)+7 of MMA group b/4, and 2^-e is stored with them.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_prep(const float* __restrict__ x, int ldx,
                                              const float* __restrict__ x2,
                                              const float* __restrict__ nw, float eps, int mode,
                                              int K, int B, float* __restrict__ xout,
                                              uint8_t* __restrict__ xprep, PrepTp tpp) {
  __shared__ __align__(16) float sv[256];
  __shared__ float red[8];
  __shared__ float mw[2][SI_ATTN_MAX_SPLITS + 1];  // mode 3: merge weights of the unit's two heads
  const int u = blockIdx.x, b = blockIdx.y, mg = b >> 2, cb = b & 3;
  const int Bm = min(4, B - 4 * mg), LW = 8 * Bm;
  const int nunit = gridDim.x;
  const int tid = threadIdx.x, k = 256 * u + tid;
  pdl_launch();  // dependents may start their independent prologue now
  // the norm weights are not written by any kernel of the step
  const float nwk = ((mode == 1 || mode == SI_PREP_RMSNORM_TP) && k < K) ? nw[k] : 0.f;
  pdl_wait();
  const float* xb = x + (int64_t)b * ldx;
  float scale = 1.f;
  float v = 0.f;
  if (mode == 3) {
    const int S = ldx, nhd = K / 128;
    const int warp = tid >> 5, lane = tid & 31;
    // this thread's first partial outputs are requested before the statistics,
    // so both arrive in one round trip
    constexpr int PRE = 48;
    const int hl0 = tid >> 7, d0 = tid & 127;
    const float* po0 = x + ((int64_t)b * nhd + 2 * u + hl0) * S * 128 + d0;
    float o0[PRE];
#pragma unroll
    for (int j = 0; j < PRE; j++) o0[j] = (k < K && j < S) ? po0[(int64_t)j * 128] : 0.f;
    if (warp < 2 && 2 * u + warp < nhd) {  // statistics of head 2u + warp
      const float2* ml = (const float2*)x2 + ((int64_t)b * nhd + 2 * u + warp) * S;
      float2 pv[(SI_ATTN_MAX_SPLITS + 32) / 32];  // all of this lane's (max, sum) pairs in one round trip
#pragma unroll
      for (int j = 0; j < (SI_ATTN_MAX_SPLITS + 32) / 32; j++)
        pv[j] = lane + 32 * j < S ? ml[lane + 32 * j] : make_float2(-INFINITY, 0.f);
      float M = -INFINITY;
#pragma unroll
      for (int j = 0; j < (SI_ATTN_MAX_SPLITS + 32) / 32; j++) M = fmaxf(M, pv[j].x);
      M = warp_max(M);
      float den = 0.f;
#pragma unroll
      for (int j = 0; j < (SI_ATTN_MAX_SPLITS + 32) / 32; j++) {
        const int s = lane + 32 * j;
        if (s < S) {
          const float w = pv[j].x == -INFINITY ? 0.f : expf(pv[j].x - M);
          mw[warp][s] = w;
          den = fmaf(w, pv[j].y, den);
        }
      }
      den = warp_sum(den);
      if (lane == 0) mw[warp][SI_ATTN_MAX_SPLITS] = 1.0f / den;
    }
    __syncthreads();
    if (k < K) {
      const float* po = po0;
      const float* wh = mw[hl0];
      float n0 = 0.f, n1 = 0.f;
#pragma unroll
      for (int j = 0; j < PRE; j += 2) {
        if (j < S) n0 = fmaf(wh[j], o0[j], n0);
        if (j + 1 < S) n1 = fmaf(wh[j + 1], o0[j + 1], n1);
      }
      for (int s0 = PRE; s0 < S; s0 += 32) {  // the rest, 32 partial outputs in flight
        float o[32];
#pragma unroll
        for (int j = 0; j < 32; j++)
          if (s0 + j < S) o[j] = po[(int64_t)(s0 + j) * 128];
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          if (s0 + j < S) n0 = fmaf(wh[s0 + j], o[j], n0);
          if (s0 + j + 1 < S) n1 = fmaf(wh[s0 + j + 1], o[j + 1], n1);
        }
      }
      v = (n0 + n1) * wh[SI_ATTN_MAX_SPLITS];
      if (xout) xout[(int64_t)b * K + k] = v;
    }
  }
  if (mode == SI_PREP_RMSNORM_TP) {
    // residual + the tp partial sums, added in rank order (identical on every
    // rank); each partial-sum element is awaited through its tag.  Four
    // elements per thread at a time, the words of every rank loaded together
    // (up to 32 loads in flight, whatever the rank count); only a word whose
    // tag is not there yet is polled.
    const unsigned want = *tpp.epoch * (unsigned)tpp.nlayers2 + (unsigned)tpp.flag_add;
    const int nper = (K + 255) / 256;  // elements of this thread: tid + 256 m
    float ss = 0.f, own = 0.f;
    const uint8_t* slot0 = tpp.comm + tpp.slots_off + (int64_t)b * tpp.ld * (int64_t)sizeof(uint2);
    for (int m0 = 0; m0 < nper; m0 += 4) {
      float a[4];
      uint2 w[SI_TP_MAX][4];
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const int i = tid + 256 * (m0 + j);
        a[j] = (m0 + j < nper && i < K) ? xb[i] : 0.f;
      }
#pragma unroll
      for (int r = 0; r < SI_TP_MAX; r++) {
        const uint2* sl = (const uint2*)(slot0 + (int64_t)r * tpp.src_stride);
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const int i = tid + 256 * (m0 + j);
          w[r][j] = (r < tpp.tp && m0 + j < nper && i < K) ? ld_tagged(sl + i) : make_uint2(0u, want);
        }
      }
#pragma unroll
      for (int r = 0; r < SI_TP_MAX; r++) {
        if (r < tpp.tp) {
          const uint2* sl = (const uint2*)(slot0 + (int64_t)r * tpp.src_stride);
#pragma unroll
          for (int j = 0; j < 4; j++) {
            const int i = tid + 256 * (m0 + j);
            if (m0 + j < nper && i < K) {
              const uint32_t bits = (int)(w[r][j].y - want) >= 0 ? w[r][j].x : wait_tagged(sl + i, want, tpp.err);
              a[j] = __fadd_rn(a[j], __uint_as_float(bits));
            }
          }
        }
      }
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const int i = tid + 256 * (m0 + j);
        if (m0 + j < nper && i < K) {
          ss = __fadd_rn(ss, __fmul_rn(a[j], a[j]));
          if (m0 + j == u) own = a[j];
        }
      }
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    float t = 0.f;
    for (int i = 0; i < 8; i++) t += red[i];
    scale = 1.0f / sqrtf(t / (float)K + eps);
    if (k < K) {
      xout[(int64_t)b * K + k] = own;
      v = __fmul_rn(__fmul_rn(own, scale), nwk);
    }
    __syncthreads();  // red is reused below
  }
  float xk = 0.f;
  if (mode == 1) {
    // sum of squares: 16-byte loads, four in flight (plus this thread's own
    // element), in the same order in every CTA of the row
    xk = k < K ? xb[k] : 0.f;
    float ss = 0.f;
    if ((K & 1023) == 0 && ((uintptr_t)xb & 15) == 0) {
      for (int i0 = 0; i0 < K; i0 += 4096) {
        float4 r[4];
#pragma unroll
        for (int j = 0; j < 4; j++)
          r[j] = i0 + 1024 * j < K ? ((const float4*)(xb + i0 + 1024 * j))[tid] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int j = 0; j < 4; j++) {
          ss = __fadd_rn(ss, __fmul_rn(r[j].x, r[j].x));
          ss = __fadd_rn(ss, __fmul_rn(r[j].y, r[j].y));
          ss = __fadd_rn(ss, __fmul_rn(r[j].z, r[j].z));
          ss = __fadd_rn(ss, __fmul_rn(r[j].w, r[j].w));
        }
      }
    } else {
      for (int i = tid; i < K; i += 256) ss = __fadd_rn(ss, __fmul_rn(xb[i], xb[i]));
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    float t = 0.f;
    for (int i = 0; i < 8; i++) t += red[i];
    scale = 1.0f / sqrtf(t / (float)K + eps);
  }
  if (k < K && mode != 3 && mode != SI_PREP_RMSNORM_TP) {
    if (mode == 1) {
      v = __fmul_rn(__fmul_rn(xk, scale), nwk);
    } else if (mode == 2) {
      const float gte = xb[k];
      const float sl = __fdiv_rn(gte, __fadd_rn(1.0f, expf(-gte)));
      v = __fmul_rn(sl, x2[(int64_t)b * ldx + k]);
    } else {
      v = xb[k];
    }
    if (xout) xout[(int64_t)b * K + k] = v;
  }
  sv[tid] = v;
  float amax = warp_max(fabsf(v));
  __syncthreads();
  if ((tid & 31) == 0) red[tid >> 5] = amax;
  __syncthreads();
  amax = 0.f;
  for (int i = 0; i < 8; i++) amax = fmaxf(amax, red[i]);
  const int e = unit_exponent(amax);
  const float s = exp2i(e);
  uint8_t* unit = xprep + xprep_off(mg, nunit, u, LW);
  if (tid < 64) {  // fragments: 8 groups x (hi, lo) x 4 lanes
    const int jj = tid >> 3, part = (tid >> 2) & 1, t = tid & 3;
    const int L = 8 * cb + 4 * part + t;
    uint32_t w[4];
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const int base = 32 * jj + 16 * h + 2 * t;
      const float v0 = sv[base] * s, v1 = sv[base + 1] * s, v2 = sv[base + 8] * s, v3 = sv[base + 9] * s;
      w[2 * h] = pack2(split_part(v0, part), split_part(v1, part));
      w[2 * h + 1] = pack2(split_part(v2, part), split_part(v3, part));
    }
    *(uint4*)(unit + (jj * LW + L) * 16) = make_uint4(w[0], w[1], w[2], w[3]);
  } else if (tid < 96) {  // warp 2: Q4_K sub-block sums (X_{2t}, X_{2t+1}) * 2^-5, and the scale
    const int lane = tid & 31;
    const float S = subblock_sum(sv, lane);
    const int part = (lane >> 2) & 1, t = lane & 3;
    const float X0 = __shfl_sync(0xFFFFFFFFu, S, 8 * t), X1 = __shfl_sync(0xFFFFFFFFu, S, 8 * t + 4);
    if (lane < 8) {
      const int L = 8 * cb + 4 * part + t;
      const float s5 = s * 0.03125f;
      *(uint32_t*)(unit + 8 * LW * 16 + L * 4) = pack2(split_part(X0 * s5, part), split_part(X1 * s5, part));
    } else if (lane == 8) {
      *(float*)(unit + 132 * LW + 4 * cb) = exp2i(-e);
    }
  }
  __syncthreads();
}

// ---------------------------------------------------------------------------
// Shared epilogue: reduce the 8 warps' partial sums and write y.
// tg/tg8: rows g and g+8 of the tile, batch 4mg + t.
// ---------------------------------------------------------------------------
template <int NMG, int EPI>
__device__ __forceinline__ void qmv_epilogue(const float (&tg)[NMG], const float (&tg8)[NMG], int B,
                                             int64_t rows, float* __restrict__ y, int tile, const TpArgs& tpa) {
  __shared__ float red[QMV_WARPS][NMG][2][32];
  __syncthreads();  // the previous tile's reduction has been read
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int mg = 0; mg < NMG; mg++) {
    red[warp][mg][0][lane] = tg[mg];
    red[warp][mg][1][lane] = tg8[mg];
  }
  __syncthreads();
  const int o = threadIdx.x;  // 2 * NMG * 32 outputs, one per thread
  if (o < 2 * NMG * 32) {
    const int mg = o >> 6, half = (o >> 5) & 1, ln = o & 31;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < QMV_WARPS; w++) v += red[w][mg][half][ln];
    const int gg = ln >> 2, tt = ln & 3;
    const int bt = 4 * mg + tt;
    const int64_t row = (int64_t)tile * 16 + gg + 8 * half;
    if (bt < B && row < rows) {
      if (EPI == SI_EPI_TP) {
        const unsigned tag = tpa.tag();
        for (int p = 0; p < tpa.tp; p++)
          st_tagged((uint2*)(tpa.peers[p] + tpa.slot_off) + (int64_t)bt * tpa.ld + row, __float_as_uint(v), tag);
      } else {
        float* dst = y + (int64_t)bt * rows + row;
        if (EPI == SI_EPI_ADD) *dst += v;
        else *dst = v;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Per-unit compute, shared by the streaming (shared memory) and the global
// memory kernels.  `Ld` reads the unit's weight bytes (w*) and this lane's
// activation data: fragments of 32-column group j (frag), the Q4_K sub-block
// sum word (xsum) and the inverse activation scale of its batch (inv).  Lanes
// without a batch column read zeros.
// ---------------------------------------------------------------------------
struct SmemLd {
  const uint8_t* w;
  const uint8_t* xf;  // lane's fragment base (or the zero region)
  const uint8_t* xs;  // lane's sub-block sum word (or zero)
  const uint8_t* xi;  // lane's inverse scale (or zero)
  int fstride;        // bytes between 32-column groups
  __device__ __forceinline__ uint4 w16(int off) const { return *(const uint4*)(w + off); }
  __device__ __forceinline__ uint2 w8(int off) const { return *(const uint2*)(w + off); }
  __device__ __forceinline__ uint32_t w4(int off) const { return *(const uint32_t*)(w + off); }
  __device__ __forceinline__ uint4 frag(int j) const { return *(const uint4*)(xf + j * fstride); }
  __device__ __forceinline__ uint32_t xsum() const { return *(const uint32_t*)xs; }
  __device__ __forceinline__ float inv() const { return *(const float*)xi; }
};

struct GlobLd {
  const uint8_t* w;
  const uint8_t* xf;
  const uint8_t* xs;
  const uint8_t* xi;
  int fstride;
  bool on, oni;
  __device__ __forceinline__ uint4 w16(int off) const { return __ldg((const uint4*)(w + off)); }
  __device__ __forceinline__ uint2 w8(int off) const { return __ldg((const uint2*)(w + off)); }
  __device__ __forceinline__ uint32_t w4(int off) const { return __ldg((const unsigned*)(w + off)); }
  __device__ __forceinline__ uint4 frag(int j) const {
    return on ? __ldg((const uint4*)(xf + j * fstride)) : make_uint4(0, 0, 0, 0);
  }
  __device__ __forceinline__ uint32_t xsum() const { return on ? __ldg((const unsigned*)xs) : 0u; }
  __device__ __forceinline__ float inv() const { return oni ? __ldg((const float*)xi) : 0.f; }
};

__device__ __forceinline__ uint32_t sc_half2(uint32_t lo4, uint32_t hi4, int s) {
  // (sc_s, sc_s) as f16x2 for sub-block s of a decoded scale pair of words.
  const uint32_t w = s < 4 ? lo4 : hi4;
  const uint32_t k = s & 3;
  const uint32_t sel = 0x5040u | k | (k << 8);
  return hsub2_u32(prmt(w, 0x64646464u, sel), 0x64006400u);
}

// One Q4_K unit (one block, 16 rows).  ld[mg] views MMA group mg.
template <int NMG, typename Ld>
__device__ __forceinline__ void unit_q4k(const Ld (&ld)[NMG], int lane, float (&tg)[NMG],
                                         float (&tg8)[NMG]) {
  const int g = lane >> 2, t = lane & 3;
  const uint4 h0 = ld[0].w16(16 * g), h1 = ld[0].w16(16 * (g + 8));
  const uint32_t scl0 = h0.y & 0x3F3F3F3Fu, mnl0 = h0.z & 0x3F3F3F3Fu;
  const uint32_t sch0 = (h0.w & 0x0F0F0F0Fu) | ((h0.y >> 2) & 0x30303030u);
  const uint32_t mnh0 = ((h0.w >> 4) & 0x0F0F0F0Fu) | ((h0.z >> 2) & 0x30303030u);
  const uint32_t scl1 = h1.y & 0x3F3F3F3Fu, mnl1 = h1.z & 0x3F3F3F3Fu;
  const uint32_t sch1 = (h1.w & 0x0F0F0F0Fu) | ((h1.y >> 2) & 0x30303030u);
  const uint32_t mnh1 = ((h1.w >> 4) & 0x0F0F0F0Fu) | ((h1.z >> 2) & 0x30303030u);
  float C[NMG][4], Cm[NMG][4];
#pragma unroll
  for (int mg = 0; mg < NMG; mg++)
#pragma unroll
    for (int i = 0; i < 4; i++) C[mg][i] = Cm[mg][i] = 0.f;
  {  // mins: A[row][k] = m_k(row) for k < 8, B[k][col] = X_k(col) * 2^-5
    const uint32_t msel = (t & 1) ? 0x5342u : 0x5140u;
    const uint32_t am0 = hsub2_u32(prmt(t < 2 ? mnl0 : mnh0, 0x64646464u, msel), 0x64006400u);
    const uint32_t am1 = hsub2_u32(prmt(t < 2 ? mnl1 : mnh1, 0x64646464u, msel), 0x64006400u);
#pragma unroll
    for (int mg = 0; mg < NMG; mg++) mma16816(Cm[mg], am0, am1, 0u, 0u, ld[mg].xsum(), 0u);
  }
#pragma unroll
  for (int c = 0; c < 4; c++) {
    const uint4 q = ld[0].w16(256 + c * 512 + lane * 16);
    uint4 xv[NMG][2];
#pragma unroll
    for (int mg = 0; mg < NMG; mg++) {
      xv[mg][0] = ld[mg].frag(2 * c);
      xv[mg][1] = ld[mg].frag(2 * c + 1);
    }
#pragma unroll
    for (int hs = 0; hs < 2; hs++) {  // sub-block s = 2c + hs
      const int s = 2 * c + hs;
      const uint32_t sg = sc_half2(scl0, sch0, s), sg8 = sc_half2(scl1, sch1, s);
#pragma unroll
      for (int kk = 0; kk < 2; kk++) {
        const int i = 2 * hs + kk;
        const uint32_t w = i == 0 ? q.x : i == 1 ? q.y : i == 2 ? q.z : q.w;
        const uint32_t w8 = w >> 8;
        // nibble masked in place = f16 subnormal q*2^-24 (16q*2^-24 for row g+8)
        const uint32_t a0 = hmul2_u32(w & 0x000F000Fu, sg);
        const uint32_t a1 = hmul2_u32(w & 0x00F000F0u, sg8);
        const uint32_t a2 = hmul2_u32(w8 & 0x000F000Fu, sg);
        const uint32_t a3 = hmul2_u32(w8 & 0x00F000F0u, sg8);
#pragma unroll
        for (int mg = 0; mg < NMG; mg++)
          mma16816(C[mg], a0, a1, a2, a3, kk ? xv[mg][hs].z : xv[mg][hs].x,
                   kk ? xv[mg][hs].w : xv[mg][hs].y);
      }
    }
  }
  const float d0 = h2f_lo(h0.x) * 16777216.f, dm0 = h2f_hi(h0.x) * 32.f;
  const float d1 = h2f_lo(h1.x) * 1048576.f, dm1 = h2f_hi(h1.x) * 32.f;
#pragma unroll
  for (int mg = 0; mg < NMG; mg++) {
    const float inv = ld[mg].inv();
    tg[mg] += inv * (d0 * (C[mg][0] + C[mg][1]) - dm0 * (Cm[mg][0] + Cm[mg][1]));
    tg8[mg] += inv * (d1 * (C[mg][2] + C[mg][3]) - dm1 * (Cm[mg][2] + Cm[mg][3]));
  }
}

__device__ __forceinline__ float sbyte(uint4 v, int k) {
  const uint32_t w = k < 4 ? v.x : k < 8 ? v.y : k < 12 ? v.z : v.w;
  return (float)(int8_t)((w >> (8 * (k & 3))) & 0xFF);
}

// One Q6_K unit (one block, 16 rows).
template <int NMG, typename Ld>
__device__ __forceinline__ void unit_q6k(const Ld (&ld)[NMG], int lane, float (&tg)[NMG],
                                         float (&tg8)[NMG]) {
  const int g = lane >> 2;
  const uint4 s0 = ld[0].w16(3072 + 16 * g), s1 = ld[0].w16(3072 + 16 * (g + 8));
  const uint32_t dp = ld[0].w4(3328 + 4 * g);
  float acc[NMG], acc8[NMG];
#pragma unroll
  for (int mg = 0; mg < NMG; mg++) acc[mg] = acc8[mg] = 0.f;
#pragma unroll
  for (int c = 0; c < 4; c++) {
    const uint4 Lq = ld[0].w16(c * 768 + lane * 16);
    const uint2 Hq = ld[0].w8(c * 768 + 512 + lane * 8);
    uint4 xv[NMG][2];
#pragma unroll
    for (int mg = 0; mg < NMG; mg++) {
      xv[mg][0] = ld[mg].frag(2 * c);
      xv[mg][1] = ld[mg].frag(2 * c + 1);
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int kt = 4 * c + i;
      const uint32_t L = i == 0 ? Lq.x : i == 1 ? Lq.y : i == 2 ? Lq.z : Lq.w;
      const uint32_t Hw = (i < 2 ? Hq.x : Hq.y) >> (2 * (i & 1));
      const uint32_t L8 = L >> 8, H8 = Hw >> 8, Hs = Hw << 8;
      const uint32_t a0 = hsub2_u32(lop3_and_or(L, 0x000F000Fu, lop3_and_or(Hw, 0x00300030u, 0x64006400u)), 0x64206420u);
      const uint32_t a1 = hsub2_u32(lop3_and_or(L, 0x00F000F0u, lop3_and_or(Hw, 0x03000300u, 0x64006400u)), 0x66006600u);
      const uint32_t a2 = hsub2_u32(lop3_and_or(L8, 0x000F000Fu, lop3_and_or(H8, 0x00300030u, 0x64006400u)), 0x64206420u);
      const uint32_t a3 = hsub2_u32(lop3_and_or(L8, 0x00F000F0u, lop3_and_or(Hs, 0x03000300u, 0x64006400u)), 0x66006600u);
      const float f0 = sbyte(s0, kt), f1 = sbyte(s1, kt);
#pragma unroll
      for (int mg = 0; mg < NMG; mg++) {
        float Cc[4] = {0.f, 0.f, 0.f, 0.f};
        const uint4& x = xv[mg][i >> 1];
        mma16816(Cc, a0, a1, a2, a3, (i & 1) ? x.z : x.x, (i & 1) ? x.w : x.y);
        acc[mg] += f0 * (Cc[0] + Cc[1]);
        acc8[mg] += f1 * (Cc[2] + Cc[3]);
      }
    }
  }
  const float d0 = h2f_lo(dp), d1 = h2f_hi(dp) * 0.0625f;
#pragma unroll
  for (int mg = 0; mg < NMG; mg++) {
    const float inv = ld[mg].inv();
    tg[mg] += inv * d0 * acc[mg];
    tg8[mg] += inv * d1 * acc8[mg];
  }
}

// One Q8_0 unit: nq (<= 8) consecutive 32-column blocks, 16 rows.
template <int NMG, typename Ld>
__device__ __forceinline__ void unit_q80(const Ld (&ld)[NMG], int lane, int nq, float (&tg)[NMG],
                                         float (&tg8)[NMG]) {
  const int g = lane >> 2;
  float acc[NMG], acc8[NMG];
#pragma unroll
  for (int mg = 0; mg < NMG; mg++) acc[mg] = acc8[mg] = 0.f;
#pragma unroll 2
  for (int qb = 0; qb < nq; qb++) {
    const uint4 q = ld[0].w16(qb * 544 + lane * 16);
    const uint32_t dp = ld[0].w4(qb * 544 + 512 + 4 * g);
    float C[NMG][4];
    uint4 xv[NMG];
#pragma unroll
    for (int mg = 0; mg < NMG; mg++) {
      C[mg][0] = C[mg][1] = C[mg][2] = C[mg][3] = 0.f;
      xv[mg] = ld[mg].frag(qb);
    }
#pragma unroll
    for (int kt = 0; kt < 2; kt++) {
      const uint32_t wg = (kt ? q.z : q.x) ^ 0x80808080u;
      const uint32_t wg8 = (kt ? q.w : q.y) ^ 0x80808080u;
      const uint32_t a0 = hsub2_u32(prmt(wg, 0x64646464u, 0x5140u), 0x64806480u);
      const uint32_t a1 = hsub2_u32(prmt(wg8, 0x64646464u, 0x5140u), 0x64806480u);
      const uint32_t a2 = hsub2_u32(prmt(wg, 0x64646464u, 0x5342u), 0x64806480u);
      const uint32_t a3 = hsub2_u32(prmt(wg8, 0x64646464u, 0x5342u), 0x64806480u);
#pragma unroll
      for (int mg = 0; mg < NMG; mg++)
        mma16816(C[mg], a0, a1, a2, a3, kt ? xv[mg].z : xv[mg].x, kt ? xv[mg].w : xv[mg].y);
    }
    const float d0 = h2f_lo(dp), d1 = h2f_hi(dp);
#pragma unroll
    for (int mg = 0; mg < NMG; mg++) {
      acc[mg] += d0 * (C[mg][0] + C[mg][1]);
      acc8[mg] += d1 * (C[mg][2] + C[mg][3]);
    }
  }
#pragma unroll
  for (int mg = 0; mg < NMG; mg++) {
    const float inv = ld[mg].inv();
    tg[mg] += inv * acc[mg];
    tg8[mg] += inv * acc8[mg];
  }
}

template <int QT>
struct QtInfo;
template <>
struct QtInfo<SI_Q4_K> { static constexpr int TBB = 2304, QPU = 1; };
template <>
struct QtInfo<SI_Q6_K> { static constexpr int TBB = 3360, QPU = 1; };
template <>
struct QtInfo<SI_Q8_0> { static constexpr int TBB = 544, QPU = 8; };

// ---------------------------------------------------------------------------
// Streaming kernel (batch 1..4, one MMA group).  One persistent CTA of NW
// warps per SM.  The units (16 rows x 256 columns) of all row tiles are
// numbered tile-major -- which is also their order in memory -- and split
// into one contiguous, equal range per warp of the grid.  Each warp streams
// its range through its own NS-deep shared-memory ring (cp.async.bulk of the
// unit's weights and prepared activations, one mbarrier per stage) and keeps
// the partial sums of the tile it is in.  A tile that lies wholly in one
// warp's range is written by that warp.  A tile split between warps leaves
// one partial per contributing warp in global scratch; the last contributor
// (per-tile arrival counter) adds them in warp order -- the result does not
// depend on timing -- and writes y.
// ---------------------------------------------------------------------------
struct QmvScratch {
  float* split;  // [tiles][maxc][64] partial sums of tiles split between warps
  int* count;    // [tiles] arrivals (zero between launches; reset by the last)
  int* err;      // device error word
  int maxc;      // contributor slots per tile
  TpArgs tp;     // SI_EPI_TP: peer slots and flags
  L2Prefetch pf; // a later kernel's weights, prefetched into L2 at launch
  int ring_mode; // k_qmv1: when the ring is filled (see the kernel)
  int q1w;       // k_qmv1 warps per CTA (16, or 8)
  PrepTp ptp;    // k_qmv1 Q1_RMSNORM_TP: the partial sums to add to the residual
  float* xout;   // ... and where CTA 0 writes the new residual
};

template <int QT, int B, int NW, int NS>
struct WarpCfg {
  static constexpr int TBB = QtInfo<QT>::TBB, QPU = QtInfo<QT>::QPU;
  static constexpr int LW = 8 * B, XB = 132 * LW + 16, WB = TBB * QPU, SB = WB + XB;
  static constexpr int ZERO = 8 * LW * 16 + 32 * 16;  // zero region (covers every lane offset)
  static constexpr int SMEM = NW * NS * SB + ZERO + NW * NS * 8;
};

template <int EPI, int B>
__device__ __forceinline__ void store_tile(float* __restrict__ y, int64_t rows, int T, int lane,
                                           float v0, float v8, const TpArgs& tpa) {
  const int g = lane >> 2, t = lane & 3;
  if (EPI == SI_EPI_TP) {  // partial rows into slot [kind][rank] of every rank, tagged
    if (t < B) {
      const int64_t r0 = (int64_t)T * 16 + g, r1 = r0 + 8;
      const unsigned tag = tpa.tag();
      for (int p = 0; p < tpa.tp; p++) {
        uint2* yb = (uint2*)(tpa.peers[p] + tpa.slot_off) + (int64_t)t * tpa.ld;
        if (r0 < rows) st_tagged(yb + r0, __float_as_uint(v0), tag);
        if (r1 < rows) st_tagged(yb + r1, __float_as_uint(v8), tag);
      }
    }
    return;
  }
  if (t < B) {
    const int64_t r0 = (int64_t)T * 16 + g, r1 = r0 + 8;
    float* yb = y + (int64_t)t * rows;
    if (r0 < rows) {
      if (EPI == SI_EPI_ADD) yb[r0] += v0;
      else yb[r0] = v0;
    }
    if (r1 < rows) {
      if (EPI == SI_EPI_ADD) yb[r1] += v8;
      else yb[r1] = v8;
    }
  }
}

template <int QT, int EPI, int B, int NW, int NS>
__global__ void __launch_bounds__(NW * 32, NW <= 8 ? 2 : 1)
    k_qmv_warp(const uint8_t* __restrict__ W, int nblk, int64_t rows, int tiles, int tile_mode,
               const uint8_t* __restrict__ xprep, float* __restrict__ y, QmvScratch scr) {
  using Cfg = WarpCfg<QT, B, NW, NS>;
  constexpr int TBB = Cfg::TBB, QPU = Cfg::QPU, LW = Cfg::LW, XB = Cfg::XB, WB = Cfg::WB, SB = Cfg::SB;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* zero = smem + NW * NS * SB;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, t = lane & 3;
  uint8_t* ring = smem + warp * NS * SB;
  const uint32_t ring_s = smem_u32(ring);
  const uint32_t bar0 = smem_u32(zero + Cfg::ZERO) + warp * NS * 8;

  const int nunit = (nblk + QPU - 1) / QPU;
  // Work split: the CTA takes units [cb, ce) -- whole row tiles in tile mode,
  // so no tile is shared between CTAs, else an even share -- and warp w the
  // w-th of NW even parts of that range.  32-bit index math (the host checks
  // tiles * nunit * grid < 2^31): a 64-bit division is a long subroutine.
  const int U = tiles * nunit;
  const int G = gridDim.x, cta = blockIdx.x;
  const int cb = tile_mode ? tiles * cta / G * nunit : U * cta / G;
  const int ce = tile_mode ? tiles * (cta + 1) / G * nunit : U * (cta + 1) / G;
  const int PC = ce - cb;
  const int ub = cb + PC * warp / NW, ue = cb + PC * (warp + 1) / NW;
  const int total = ue - ub;

  for (int i = threadIdx.x; i < Cfg::ZERO / 4; i += blockDim.x) ((uint32_t*)zero)[i] = 0u;
  if (lane == 0) {
    for (int s = 0; s < NS; s++) mbar_init(bar0 + 8 * s, 1);
    mbar_fence_init();
  }
  __syncthreads();  // zero region and barriers ready

  // Units are contiguous in memory in range order, so the weight cursor only
  // advances; the activation cursor wraps to unit 0 at each tile.
  const int c0T = ub / nunit;
  const int c0U = ub - c0T * nunit;
  const uint8_t* wsrc = W + ((int64_t)c0T * nblk + (int64_t)c0U * QPU) * TBB;
  int iU = c0U;                      // unit index (in its tile) of the next copy to issue
  const int pre = total < NS ? total : NS;
  const uint64_t pol = l2_evict_first_policy();  // weights are read once per step
  if (lane == 0) {
    const uint8_t* p = wsrc;
    int u = c0U;
    for (int s = 0; s < pre; s++) {
      const uint32_t wb = (uint32_t)(min(QPU, nblk - u * QPU) * TBB);
      mbar_expect_tx(bar0 + 8 * s, wb);
      bulk_g2s_ef(ring_s + s * SB, p, wb, bar0 + 8 * s, pol);
      p += wb;
      if (++u == nunit) u = 0;
    }
  }
  l2_prefetch_share(scr.pf);
  pdl_launch();  // dependents may start their independent prologue now
  pdl_wait();
  if (lane == 0) {
    int u = c0U;
    for (int s = 0; s < pre; s++) {
      mbar_arrive_expect_tx(bar0 + 8 * s, XB);
      bulk_g2s(ring_s + s * SB + WB, xprep + (int64_t)u * XB, XB, bar0 + 8 * s);
      if (++u == nunit) u = 0;
    }
  }
  for (int s = 0; s < pre; s++) {
    wsrc += (min(QPU, nblk - iU * QPU) * TBB);
    if (++iU == nunit) iU = 0;
  }
  int issued = pre;

  const bool on = lane < LW, oni = 8 * t < LW;
  const int xf_off = on ? WB + lane * 16 : -1;  // -1: read the zero region
  float tg[1] = {0.f}, tg8[1] = {0.f};
  float p0a = 0.f, p0b = 0.f, p1a = 0.f, p1b = 0.f;  // partials of the shared first / last tile
  bool has0 = false, has1 = false;
  bool ok = true;
  // pend: stages with a copy in flight; par: the phase each completes next.
  // After a wait gives up the warp issues nothing more and waits (bounded)
  // only once on each stage still in flight.
  uint32_t pend = (1u << pre) - 1u, par = 0u;
  int cT = c0T, cU = c0U;
  int left = min(nunit - c0U, total);  // units of the current tile in this range
  int tile_first = c0T * nunit;
  for (int k0 = 0; k0 < total && ok; k0 += NS) {
#pragma unroll
    for (int s = 0; s < NS; s++) {
      if (k0 + s >= total) break;
      if (!__all_sync(0xFFFFFFFFu, mbar_wait_bounded(bar0 + 8 * s, (par >> s) & 1u))) {
        if (lane == 0) atomicOr(scr.err, SI_DEVERR_WAIT_TIMEOUT);
        ok = false;
        break;
      }
      pend &= ~(1u << s);
      par ^= 1u << s;
      {
        const uint8_t* st = ring + s * SB;
        SmemLd ld[1];
        ld[0].w = st;
        ld[0].xf = xf_off >= 0 ? st + xf_off : zero + lane * 16;
        ld[0].xs = on ? st + WB + 8 * LW * 16 + lane * 4 : zero;
        ld[0].xi = oni ? st + WB + 132 * LW + 4 * t : zero;
        ld[0].fstride = LW * 16;
        if (QT == SI_Q4_K) unit_q4k<1>(ld, lane, tg, tg8);
        else if (QT == SI_Q6_K) unit_q6k<1>(ld, lane, tg, tg8);
        else unit_q80<1>(ld, lane, min(QPU, nblk - cU * QPU), tg, tg8);
      }
      __syncwarp();
      if (issued < total) {  // refill this stage with the next unit of the range
        const uint32_t wb = (uint32_t)(min(QPU, nblk - iU * QPU) * TBB);
        if (lane == 0) {
          mbar_arrive_expect_tx(bar0 + 8 * s, wb + XB);
          bulk_g2s_ef(ring_s + s * SB, wsrc, wb, bar0 + 8 * s, pol);
          bulk_g2s(ring_s + s * SB + WB, xprep + (int64_t)iU * XB, XB, bar0 + 8 * s);
        }
        wsrc += wb;
        if (++iU == nunit) iU = 0;
        issued++;
        pend |= 1u << s;
      }
      cU++;
      if (--left == 0) {
        // ---- this warp's part of tile cT is done ----
        const int t0 = tile_first, t1 = tile_first + nunit;  // tile's unit range
        if (t0 >= ub && t1 <= ue) {
          store_tile<EPI, B>(y, rows, cT, lane, tg[0], tg8[0], scr.tp);
        } else if (cT == c0T) {  // first tile of the range, shared with other warps
          p0a = tg[0];
          p0b = tg8[0];
          has0 = true;
        } else {  // last tile of the range, shared
          p1a = tg[0];
          p1b = tg8[0];
          has1 = true;
        }
        tg[0] = tg8[0] = 0.f;
        cU = 0;
        cT++;
        tile_first += nunit;
        left = min(nunit, total - (k0 + s) - 1);
      }
    }
  }
  if (!ok) mbar_drain(bar0, pend, par, NS);
  // ---- tiles shared between warps ----
  // Every warp has drained its ring; the ring memory now holds each warp's (at
  // most two) shared-tile partials.  The first contributor of a tile inside
  // this CTA adds the CTA's partials in warp order.  A tile that also spans
  // other CTAs goes through global scratch: one slot per CTA, and the last
  // CTA to arrive (per-tile counter) adds the slots in CTA order.  The result
  // does not depend on timing.
  __syncthreads();
  float* part = (float*)smem;  // [NW][2][64]
  part[(warp * 2 + 0) * 64 + lane] = p0a;
  part[(warp * 2 + 0) * 64 + 32 + lane] = p0b;
  part[(warp * 2 + 1) * 64 + lane] = p1a;
  part[(warp * 2 + 1) * 64 + 32 + lane] = p1b;
  __syncthreads();
  auto warp_of = [&](int q) { return ((q - cb + 1) * NW - 1) / PC; };  // warp holding unit q
#pragma unroll 1
  for (int sl = 0; sl < 2; sl++) {
    if (!(sl == 0 ? has0 : has1) || !ok) continue;
    const int T = sl == 0 ? c0T : cT - 1;
    const int t0 = T * nunit, t1 = t0 + nunit;
    const int lo = t0 > cb ? t0 : cb, hi = t1 < ce ? t1 : ce;  // the tile's part in this CTA
    const int jf = warp_of(lo), jl = warp_of(hi - 1);
    if (warp != jf) continue;  // another warp of this CTA combines this tile
    float a = 0.f, b8 = 0.f;
    for (int j = jf; j <= jl; j++) {
      const int fj = cb + PC * j / NW;                    // first unit of warp j
      const int slot = (fj >= t0 && fj < t1) ? 0 : 1;  // T is warp j's first tile?
      a += part[(j * 2 + slot) * 64 + lane];
      b8 += part[(j * 2 + slot) * 64 + 32 + lane];
    }
    if (t0 >= cb && t1 <= ce) {  // the whole tile is in this CTA
      store_tile<EPI, B>(y, rows, T, lane, a, b8, scr.tp);
      continue;
    }
    // unit x lies in CTA ((x + 1) G - 1) / U (even-share mode only)
    const int cf = ((t0 + 1) * G - 1) / U, cl = (t1 * G - 1) / U;
    const int ncon = cl - cf + 1, cslot = cta - cf;
    float* base = scr.split + (int64_t)T * scr.maxc * 64;
    base[cslot * 64 + lane] = a;
    base[cslot * 64 + 32 + lane] = b8;
    __threadfence();
    __syncwarp();
    int prev = 0;
    if (lane == 0) prev = atomicAdd(scr.count + T, 1);
    prev = __shfl_sync(0xFFFFFFFFu, prev, 0);
    if (prev == ncon - 1) {  // last CTA: add the slots in CTA order
      __threadfence();
      float va[8], vb[8];
      float sa = 0.f, sb = 0.f;
      for (int j0 = 0; j0 < ncon; j0 += 8) {
        const int nj = ncon - j0 < 8 ? ncon - j0 : 8;
#pragma unroll
        for (int j = 0; j < 8; j++)
          if (j < nj) {
            va[j] = __ldcg(base + (j0 + j) * 64 + lane);
            vb[j] = __ldcg(base + (j0 + j) * 64 + 32 + lane);
          }
#pragma unroll
        for (int j = 0; j < 8; j++)
          if (j < nj) {
            sa += va[j];
            sb += vb[j];
          }
      }
      store_tile<EPI, B>(y, rows, T, lane, sa, sb, scr.tp);
      if (lane == 0) scr.count[T] = 0;
    }
  }
}

// ---------------------------------------------------------------------------
// Batch-1 Q4_K kernel.  Same persistent layout as k_qmv_warp (148 CTAs, per-
// warp contiguous ranges, deterministic split-tile combine), with three
// changes that cut the instructions per unit roughly in half:
//  * the whole prepared activation vector is copied into shared memory once
//    per CTA, so the ring carries only weights, two units per stage in one
//    bulk copy;
//  * the sub-block scales are applied after the MMA: k-tiles of sub-block s
//    accumulate into MMA column 2(s%4) (hi) / 2(s%4)+1 (lo) -- the lanes of
//    that column class supply the activation fragment, the others zeros --
//    and sub-blocks 0-3 and 4-7 use two accumulators, so lane (g, t) ends a
//    unit holding the partial sums of sub-blocks t and t+4 of rows g and g+8
//    and scales them by sc * d once (the nibbles go to the MMA unscaled);
//  * shared-memory offsets are 32-bit.
// Rows g+8 read their nibbles from bits 4-7 (16 q), compensated in d.
// ---------------------------------------------------------------------------
struct Q1Cfg {
  static constexpr int US = 2, TBB = 2304, SB = US * TBB;  // bytes per ring stage
  static constexpr int XB = 132 * 8 + 16;                   // prepared bytes per column unit
  static constexpr int ZERO = 1024;                         // zero fragments: 8 groups x 128 B
  // ring | zero fragments | activations | barriers | f32 [64] reduction |
  // partial sums [NW][2][64] f32 after the main loop, sharing their space with
  // the f32 staging (nunit * 256) of a fused RmsNorm before it
  __host__ __device__ static size_t red_off(int NW, int NS, int nunit) {
    return ((size_t)NW * NS * SB + ZERO + (size_t)nunit * XB + (size_t)(NW * NS + 1) * 8 + 15) & ~(size_t)15;
  }
  __host__ __device__ static size_t part_off(int NW, int NS, int nunit) { return red_off(NW, NS, nunit) + 256; }
  static size_t smem(int NW, int NS, int nunit, int pmode) {
    const size_t part = (size_t)NW * 2 * 64 * 4;
    const size_t stage = (pmode == 1 || pmode == 3) ? (size_t)nunit * 256 * 4 : pmode == 2 ? (size_t)NW * 256 * 4 : 0;
    return part_off(NW, NS, nunit) + (part > stage ? part : stage);
  }
};

// Input preparation of a k_qmv1 launch: 0 = prepared units copied from
// xprep, 1 = RmsNorm of x (q1_rms_prep).
// 2 = SiLU(gate) * up of two f32 inputs (q1_silu_prep).
// 3 = RmsNorm of the residual plus every rank's tensor-parallel partial sums
// (SI_PREP_RMSNORM_TP's arithmetic); CTA 0 also writes the new residual.
enum { Q1_PREPARED = 0, Q1_RMSNORM = 1, Q1_SILU = 2, Q1_RMSNORM_TP = 3 };
constexpr int Q1_SILU_MAX_UNITS = 64;  // 4 units per warp of 16

// ld_tagged without a compiler memory barrier, so the residual's loads and
// these can be in flight together (the words are only read, and each is
// single-copy atomic).
__device__ __forceinline__ uint2 ld_tagged_free(const void* p) {
  uint64_t w;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p));
  return make_uint2((uint32_t)w, (uint32_t)(w >> 32));
}

// Fused RmsNorm + activation preparation of a batch-1 k_qmv1 launch: every
// CTA reads the whole input x (K <= NW * 512 columns, 4 x 16-byte loads per
// thread; nwv holds this thread's norm weights, read before the dependency
// wait) and packs x * w into its prepared units in shared memory as k_prep
// does.  RmsNorm (TensorOps.RmsNorm, TensorOps.cs:135-145) multiplies every
// element by one scale, 1 / sqrtf(ss / n + eps); it is returned here and
// applied to the matvec's outputs, so packing starts without waiting for the
// sum of squares (the same products, rounded in another order: ~1e-7).  The
// sum of squares is taken in the same order by every CTA.
template <int NW, bool TPSUM>
__device__ __forceinline__ float q1_rms_prep(const float* __restrict__ xf, const float4 (&nwv)[4], float eps,
                                             int nunit, float* red, float* stage, uint8_t* xs,
                                             const PrepTp& tpp, float* __restrict__ xout) {
  constexpr int XB = Q1Cfg::XB;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, K = nunit * 256;
  float4 xv[4];
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const int i = 4 * tid + NW * 128 * j;
    xv[j] = i < K ? __ldcg((const float4*)(xf + i)) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if constexpr (TPSUM) {
    // residual + the ranks' partial sums in rank order, as SI_PREP_RMSNORM_TP
    // adds them; each word awaited through its tag.  The words of all 16
    // elements of two ranks are requested together (one round trip per two
    // ranks: these system-scope loads are slow).
    const unsigned want = *tpp.epoch * (unsigned)tpp.nlayers2 + (unsigned)tpp.flag_add;
    const uint8_t* slot0 = tpp.comm + tpp.slots_off;
    float a[4][4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      a[j][0] = xv[j].x;
      a[j][1] = xv[j].y;
      a[j][2] = xv[j].z;
      a[j][3] = xv[j].w;
    }
    for (int r0 = 0; r0 < tpp.tp; r0 += 2) {
      uint2 w[2][4][4];
#pragma unroll
      for (int r = 0; r < 2; r++)
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const int i = 4 * tid + NW * 128 * j;
#pragma unroll
          for (int e = 0; e < 4; e++)
            w[r][j][e] = r0 + r < tpp.tp && i < K
                             ? ld_tagged_free((const uint2*)(slot0 + (int64_t)(r0 + r) * tpp.src_stride) + i + e)
                             : make_uint2(0u, want);
        }
#pragma unroll
      for (int r = 0; r < 2; r++) {
        if (r0 + r >= tpp.tp) break;
        const uint2* sl = (const uint2*)(slot0 + (int64_t)(r0 + r) * tpp.src_stride);
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const int i = 4 * tid + NW * 128 * j;
          if (i >= K) continue;
#pragma unroll
          for (int e = 0; e < 4; e++) {
            const uint32_t bits =
                (int)(w[r][j][e].y - want) >= 0 ? w[r][j][e].x : wait_tagged(sl + i + e, want, tpp.err);
            a[j][e] = __fadd_rn(a[j][e], __uint_as_float(bits));
          }
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int i = 4 * tid + NW * 128 * j;
      xv[j] = make_float4(a[j][0], a[j][1], a[j][2], a[j][3]);
      if (blockIdx.x == 0 && i < K) *(float4*)(xout + i) = xv[j];
    }
  }
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const int i = 4 * tid + NW * 128 * j;
    if (i < K)
      *(float4*)(stage + i) = make_float4(__fmul_rn(xv[j].x, nwv[j].x), __fmul_rn(xv[j].y, nwv[j].y),
                                          __fmul_rn(xv[j].z, nwv[j].z), __fmul_rn(xv[j].w, nwv[j].w));
  }
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 4; j++) {
    ss = __fadd_rn(ss, __fmul_rn(xv[j].x, xv[j].x));
    ss = __fadd_rn(ss, __fmul_rn(xv[j].y, xv[j].y));
    ss = __fadd_rn(ss, __fmul_rn(xv[j].z, xv[j].z));
    ss = __fadd_rn(ss, __fmul_rn(xv[j].w, xv[j].w));
  }
  ss = warp_sum(ss);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  for (int u = warp; u < nunit; u += NW)  // one warp per 256-column unit
    pack_unit_warp(stage + 256 * u, xs + u * XB, 8, 0, lane);
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < NW; w++) tot += red[w];
  return 1.0f / sqrtf(tot / (float)K + eps);
}

// Fused SiLU * up + activation preparation of a batch-1 k_qmv1 launch (the
// down projection's input): v = SiLU(gate) * up (TensorOps.SiLU then
// MulInPlace, TensorOps.cs:191-195, :169-185, in k_prep's arithmetic), one
// warp per 256-column unit with all of the warp's loads (<= 4 units) issued
// before any is used; each unit is packed exactly as k_prep does.  stage:
// 1 KB per warp.
template <int NW>
__device__ __forceinline__ void q1_silu_prep(const float* __restrict__ gate, const float* __restrict__ up, int nunit,
                                             float* stage, uint8_t* xs) {
  constexpr int XB = Q1Cfg::XB, MAXU = 4;  // units per warp (the launcher caps nunit at 4 NW)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* sv = stage + warp * 256;
  float4 g[MAXU][2], u[MAXU][2];
#pragma unroll
  for (int i = 0; i < MAXU; i++) {
    const int un = warp + NW * i;
#pragma unroll
    for (int j = 0; j < 2; j++) {
      g[i][j] = un < nunit ? __ldcg((const float4*)(gate + 256 * un) + 2 * lane + j) : make_float4(0.f, 0.f, 0.f, 0.f);
      u[i][j] = un < nunit ? __ldcg((const float4*)(up + 256 * un) + 2 * lane + j) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  auto sm = [](float gv, float uv) { return __fmul_rn(__fdiv_rn(gv, __fadd_rn(1.0f, expf(-gv))), uv); };
#pragma unroll
  for (int i = 0; i < MAXU; i++) {
    const int un = warp + NW * i;
    if (un >= nunit) break;
#pragma unroll
    for (int j = 0; j < 2; j++)
      *(float4*)(sv + 8 * lane + 4 * j) = make_float4(sm(g[i][j].x, u[i][j].x), sm(g[i][j].y, u[i][j].y),
                                                      sm(g[i][j].z, u[i][j].z), sm(g[i][j].w, u[i][j].w));
    __syncwarp();
    pack_unit_warp(sv, xs + un * XB, 8, 0, lane);
    __syncwarp();
  }
  __syncthreads();
}

__device__ __forceinline__ float red4(float v) {
  v += __shfl_xor_sync(0xFFFFFFFFu, v, 1);
  return v + __shfl_xor_sync(0xFFFFFFFFu, v, 2);
}

// exact small integer -> f32: 2^23 + v as bits, minus 2^23
__device__ __forceinline__ float magic_f(uint32_t bits) { return __uint_as_float(bits) - 8388608.f; }

template <int EPI, int NW, int NS, bool TPSUM>
__global__ void __launch_bounds__(NW * 32, NW <= 8 ? 2 : 1)
    k_qmv1(const uint8_t* __restrict__ W, int nunit, int64_t rows, int tiles, int tile_mode,
           int pmode, const uint8_t* __restrict__ xprep, const float* __restrict__ xf, const float* __restrict__ nw,
           float eps, float* __restrict__ y, QmvScratch scr) {
  constexpr int SB = Q1Cfg::SB, TBB = Q1Cfg::TBB, XB = Q1Cfg::XB;
  constexpr int RING = NW * NS * SB;
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  uint8_t* const ring = smem + warp * NS * SB;
  const uint8_t* const zero = smem + RING;
  const uint8_t* const xs = zero + Q1Cfg::ZERO;
  const uint32_t bar_x = smem_u32(xs + nunit * XB);
  const uint32_t bar0 = bar_x + 8 + warp * NS * 8;

  // Work split: the CTA takes pairs [cb, ce) -- whole row tiles in tile
  // mode, so no tile is shared between CTAs, else an even share of all
  // pairs -- and warp w of the CTA the w-th of NW even parts of that range.
  // Pair and unit indices fit in 32 bits (the host checks tiles * nunit
  // < 2^24, so products with the grid size stay below 2^31); a 32-bit
  // division is a short sequence, a 64-bit one a long subroutine.
  const int P = tiles * nunit / 2;  // unit pairs
  const int npt = nunit / 2;        // pairs per tile
  const int G = gridDim.x, cta = blockIdx.x;
  const int cb = tile_mode ? tiles * cta / G * npt : P * cta / G;
  const int ce = tile_mode ? tiles * (cta + 1) / G * npt : P * (cta + 1) / G;
  const int PC = ce - cb;
  const int pb = cb + PC * warp / NW, pe = cb + PC * (warp + 1) / NW;
  const int npair = pe - pb;
  const int ub = 2 * pb;

  for (int i = threadIdx.x; i < Q1Cfg::ZERO / 16; i += blockDim.x) ((uint4*)(smem + RING))[i] = make_uint4(0, 0, 0, 0);
  if (threadIdx.x == 0) mbar_init(bar_x, 1);
  if (lane == 0)
    for (int s = 0; s < NS; s++) mbar_init(bar0 + 8 * s, 1);
  mbar_fence_init();
  __syncthreads();
  const uint8_t* wsrc = W + (int64_t)ub * TBB;  // units are contiguous in range order
  // One ring stage per warp is requested before the dependency wait, the
  // rest once the activations are in: requests queued ahead of the
  // activation loads delay them (the loads wait behind up to one stage per
  // warp of weight bytes instead of the whole ring).
  // When the ring is filled (scr.ring_mode):
  //  0  one stage per warp before the dependency wait, the rest once the input
  //     is prepared: bulk copies queued ahead of the input's own copy delay it
  //  1  the whole ring before the dependency wait; prepared input through
  //     ordinary loads
  //  2  the warp's whole weight range prefetched into L2 before the wait, the
  //     ring filled once the input is prepared (ordinary loads for it)
  const int pre = npair < NS ? npair : NS;
  const uint64_t pol = l2_evict_first_policy();  // weights are read once per step
  const int rmode = scr.ring_mode;
  auto issue_stages = [&](int s0, int s1) {
    if (lane == 0)
      for (int s = s0; s < s1; s++) {
        mbar_arrive_expect_tx(bar0 + 8 * s, SB);
        bulk_g2s_ef(smem_u32(ring + s * SB), wsrc + s * SB, SB, bar0 + 8 * s, pol);
      }
  };
  if (rmode == 2) {
    if (lane == 0)
      for (uint32_t o = 0, n = (uint32_t)npair * SB; o < n; o += 65536u)
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(wsrc + o), "r"(min(65536u, n - o))
                     : "memory");
  } else {
    issue_stages(0, rmode == 1 ? pre : min(pre, 1));
  }
  l2_prefetch_share(scr.pf);
  pdl_launch();  // dependents may start their independent prologue now
  // pmode: prepared units in xprep, or the f32 input xf normalised here
  // with weights nw
  float4 nwv[4];
  if (pmode == Q1_RMSNORM || pmode == Q1_RMSNORM_TP) {
#pragma unroll
    for (int j = 0; j < 4; j++) {  // norm weights: not written by any kernel of the step
      const int i = 4 * (int)threadIdx.x + NW * 128 * j;
      nwv[j] = i < nunit * 256 ? *(const float4*)(nw + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  pdl_wait();
  bool ok = true;
  float oscale = 1.f;  // RmsNorm's scale, applied to the outputs
  if (pmode == Q1_SILU) {  // xf: gate, nw: up
    q1_silu_prep<NW>(xf, nw, nunit, (float*)(smem + Q1Cfg::part_off(NW, NS, nunit)), (uint8_t*)xs);
  } else if (pmode != Q1_PREPARED) {
    if constexpr (TPSUM)
      oscale = q1_rms_prep<NW, true>(xf, nwv, eps, nunit, (float*)(smem + Q1Cfg::red_off(NW, NS, nunit)),
                                     (float*)(smem + Q1Cfg::part_off(NW, NS, nunit)), (uint8_t*)xs, scr.ptp, scr.xout);
    else
      oscale = q1_rms_prep<NW, false>(xf, nwv, eps, nunit, (float*)(smem + Q1Cfg::red_off(NW, NS, nunit)),
                                      (float*)(smem + Q1Cfg::part_off(NW, NS, nunit)), (uint8_t*)xs, scr.ptp,
                                      scr.xout);
  } else if (rmode == 0) {
    if (threadIdx.x == 0) {
      mbar_arrive_expect_tx(bar_x, (uint32_t)(nunit * XB));
      bulk_g2s(smem_u32(xs), xprep, (uint32_t)(nunit * XB), bar_x);
    }
    ok = mbar_wait_bounded(bar_x, 0);
    if (!ok && lane == 0) atomicOr(scr.err, SI_DEVERR_WAIT_TIMEOUT);
  } else {
    // prepared units (nunit * XB bytes, a multiple of 16), 16 bytes per load
    // with up to four loads in flight per thread
    const int n16 = nunit * XB / 16;
    for (int i0 = threadIdx.x; i0 < n16; i0 += 4 * NW * 32) {
      uint4 v[4];
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const int i = i0 + j * NW * 32;
        if (i < n16) v[j] = __ldcg((const uint4*)xprep + i);
      }
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const int i = i0 + j * NW * 32;
        if (i < n16) ((uint4*)xs)[i] = v[j];
      }
    }
    __syncthreads();
  }
  if (rmode == 0) issue_stages(1, pre);
  else if (rmode == 2) issue_stages(0, pre);

  // per-lane constants
  const int cls = lane >> 3;                                   // MMA column class
  const int xl = (lane & 7) * 16;                              // fragment slot in a group
  const int sh = 8 * t;                                        // byte of sub-blocks t, t+4
  const uint32_t msel = (t & 1) ? 0x5342u : 0x5140u;
  const uint8_t* const xsum0 = lane < 8 ? xs + 1024 + lane * 4 : zero;
  const int xsum_step = lane < 8 ? XB : 0;

  float tg = 0.f, tg8 = 0.f;
  float p0a = 0.f, p0b = 0.f, p1a = 0.f, p1b = 0.f;
  bool has0 = false, has1 = false;
  const int c0T = ub / nunit;
  int cT = c0T;
  int cU = ub - c0T * nunit;  // even
  const bool first_partial = cU != 0;

  auto unit = [&](const uint8_t* st, int cu) {
    const uint8_t* xu = xs + cu * XB;
    const uint4 h0 = *(const uint4*)(st + 16 * g), h1 = *(const uint4*)(st + 16 * (g + 8));
    const uint8_t* xb[4];
#pragma unroll
    for (int c = 0; c < 4; c++) xb[c] = c == cls ? xu + xl : zero;
    // mins: A[row][k] = m_k(row) (k < 8), B[k][col] = X_k(col) * 2^-5 in columns 0 (hi), 1 (lo)
    const uint32_t mnl0 = h0.z & 0x3F3F3F3Fu, mnh0 = ((h0.w >> 4) & 0x0F0F0F0Fu) | ((h0.z >> 2) & 0x30303030u);
    const uint32_t mnl1 = h1.z & 0x3F3F3F3Fu, mnh1 = ((h1.w >> 4) & 0x0F0F0F0Fu) | ((h1.z >> 2) & 0x30303030u);
    const uint32_t am0 = hsub2_u32(prmt(t < 2 ? mnl0 : mnh0, 0x64646464u, msel), 0x64006400u);
    const uint32_t am1 = hsub2_u32(prmt(t < 2 ? mnl1 : mnh1, 0x64646464u, msel), 0x64006400u);
    float Cm[4] = {0.f, 0.f, 0.f, 0.f}, C0[4] = {0.f, 0.f, 0.f, 0.f}, C1[4] = {0.f, 0.f, 0.f, 0.f};
    mma16816(Cm, am0, am1, 0u, 0u, *(const uint32_t*)(xsum0 + cu * xsum_step), 0u);
#pragma unroll
    for (int c = 0; c < 4; c++) {
      const uint4 q = *(const uint4*)(st + 256 + c * 512 + lane * 16);
#pragma unroll
      for (int hs = 0; hs < 2; hs++) {
        const int jj = 2 * c + hs;  // sub-block
        const uint4 xv = *(const uint4*)(xb[jj & 3] + jj * 128);
#pragma unroll
        for (int kk = 0; kk < 2; kk++) {
          const int i = 2 * hs + kk;
          const uint32_t w = i == 0 ? q.x : i == 1 ? q.y : i == 2 ? q.z : q.w;
          const uint32_t w8 = w >> 8;
          float* acc = jj < 4 ? C0 : C1;
          mma16816(acc, w & 0x000F000Fu, w & 0x00F000F0u, w8 & 0x000F000Fu, w8 & 0x00F000F0u,
                   kk ? xv.z : xv.x, kk ? xv.w : xv.y);
        }
      }
    }
    // scales of sub-blocks t and t+4 (GetScaleMinK4), rows g and g+8
    const uint32_t ys0 = h0.y >> sh, ws0 = h0.w >> sh, ys1 = h1.y >> sh, ws1 = h1.w >> sh;
    const float sa0 = magic_f(lop3_and_or(ys0, 0x3Fu, 0x4B000000u));
    const float sb0 = magic_f(lop3_and_or(ws0, 0x0Fu, lop3_and_or(ys0 >> 2, 0x30u, 0x4B000000u)));
    const float sa1 = magic_f(lop3_and_or(ys1, 0x3Fu, 0x4B000000u));
    const float sb1 = magic_f(lop3_and_or(ws1, 0x0Fu, lop3_and_or(ys1 >> 2, 0x30u, 0x4B000000u)));
    const float inv = *(const float*)(xu + 1056);
    const float d0 = h2f_lo(h0.x) * (16777216.f * inv), dm0 = h2f_hi(h0.x) * (32.f * inv);
    const float d1 = h2f_lo(h1.x) * (1048576.f * inv), dm1 = h2f_hi(h1.x) * (32.f * inv);
    tg += d0 * (sa0 * (C0[0] + C0[1]) + sb0 * (C1[0] + C1[1])) - dm0 * (Cm[0] + Cm[1]);
    tg8 += d1 * (sa1 * (C0[2] + C0[3]) + sb1 * (C1[2] + C1[3])) - dm1 * (Cm[2] + Cm[3]);
  };

  // pend: stages with a copy in flight; par: the phase each completes next.
  // After a wait gives up the warp issues nothing more and waits (bounded)
  // only once on each stage still in flight.
  uint32_t pend = (1u << pre) - 1u, par = 0u;
  for (int k0 = 0; k0 < npair && ok; k0 += NS) {
#pragma unroll
    for (int s = 0; s < NS; s++) {
      const int k = k0 + s;
      if (k >= npair) break;
      if (!__all_sync(0xFFFFFFFFu, mbar_wait_bounded(bar0 + 8 * s, (par >> s) & 1u))) {
        if (lane == 0) atomicOr(scr.err, SI_DEVERR_WAIT_TIMEOUT);
        ok = false;
        break;
      }
      pend &= ~(1u << s);
      par ^= 1u << s;
      uint8_t* st = ring + s * SB;
      unit(st, cU);
      unit(st + TBB, cU + 1);
      __syncwarp();
      if (k + NS < npair) {  // refill this stage with pair k + NS
        if (lane == 0) {
          mbar_arrive_expect_tx(bar0 + 8 * s, SB);
          bulk_g2s_ef(smem_u32(st), wsrc + (int64_t)(k + NS) * SB, SB, bar0 + 8 * s, pol);
        }
        pend |= 1u << s;
      }
      cU += 2;
      if (cU == nunit) {  // this warp's part of tile cT is done
        const float a = red4(tg), b8 = red4(tg8);
        if (cT == c0T && first_partial) {
          p0a = a;
          p0b = b8;
          has0 = true;
        } else {
          store_tile<EPI, 1>(y, rows, cT, lane, a * oscale, b8 * oscale, scr.tp);
        }
        tg = tg8 = 0.f;
        cU = 0;
        cT++;
      }
    }
  }
  if (!ok) mbar_drain(bar0, pend, par, NS);
  const int T1 = cT;
  if (cU != 0 && npair > 0) {  // the range ends inside tile cT
    const float a = red4(tg), b8 = red4(tg8);
    if (cT == c0T && first_partial) {
      p0a = a;
      p0b = b8;
      has0 = true;
    } else {
      p1a = a;
      p1b = b8;
      has1 = true;
    }
  }
  // ---- tiles shared between warps of this CTA, then between CTAs ----
  __syncthreads();
  float* part = (float*)(smem + Q1Cfg::part_off(NW, NS, nunit));  // [NW][2][64], apart from the ring
  part[(warp * 2 + 0) * 64 + lane] = p0a;
  part[(warp * 2 + 0) * 64 + 32 + lane] = p0b;
  part[(warp * 2 + 1) * 64 + lane] = p1a;
  part[(warp * 2 + 1) * 64 + 32 + lane] = p1b;
  __syncthreads();
  auto warp_of = [&](int q) { return ((q - cb + 1) * NW - 1) / PC; };  // warp holding pair q
#pragma unroll 1
  for (int sl = 0; sl < 2; sl++) {
    if (!(sl == 0 ? has0 : has1) || !ok) continue;
    const int T = sl == 0 ? c0T : T1;
    const int q0 = T * npt, q1 = q0 + npt;  // tile's pair range
    const int lo = q0 > cb ? q0 : cb, hi = q1 < ce ? q1 : ce;  // its part in this CTA
    const int jf = warp_of(lo), jl = warp_of(hi - 1);
    if (warp != jf) continue;
    float a = 0.f, b8 = 0.f;
    const int u0 = T * nunit, u1 = u0 + nunit;  // tile's unit range
    for (int j = jf; j <= jl; j++) {
      const int fj = 2 * (cb + PC * j / NW);  // first unit of warp j
      const int slot = (fj > u0 && fj < u1) ? 0 : 1;  // it starts inside T: partial 0
      a += part[(j * 2 + slot) * 64 + lane];
      b8 += part[(j * 2 + slot) * 64 + 32 + lane];
    }
    if (q0 >= cb && q1 <= ce) {  // the whole tile is in this CTA
      store_tile<EPI, 1>(y, rows, T, lane, a * oscale, b8 * oscale, scr.tp);
      continue;
    }
    // pair p lies in CTA ((p + 1) G - 1) / P (even-share mode only)
    const int cf = ((q0 + 1) * G - 1) / P, cl = (q1 * G - 1) / P;
    const int ncon = cl - cf + 1, cslot = cta - cf;
    float* base = scr.split + (int64_t)T * scr.maxc * 64;
    base[cslot * 64 + lane] = a;
    base[cslot * 64 + 32 + lane] = b8;
    __threadfence();
    __syncwarp();
    int prev = 0;
    if (lane == 0) prev = atomicAdd(scr.count + T, 1);
    prev = __shfl_sync(0xFFFFFFFFu, prev, 0);
    if (prev == ncon - 1) {
      __threadfence();
      float sa = 0.f, sb = 0.f;
      for (int j0 = 0; j0 < ncon; j0 += 8) {
        float va[8], vb[8];
        const int nj = ncon - j0 < 8 ? ncon - j0 : 8;
#pragma unroll
        for (int j = 0; j < 8; j++)
          if (j < nj) {
            va[j] = __ldcg(base + (j0 + j) * 64 + lane);
            vb[j] = __ldcg(base + (j0 + j) * 64 + 32 + lane);
          }
#pragma unroll
        for (int j = 0; j < 8; j++)
          if (j < nj) {
            sa += va[j];
            sb += vb[j];
          }
      }
      store_tile<EPI, 1>(y, rows, T, lane, sa * oscale, sb * oscale, scr.tp);
      if (lane == 0) scr.count[T] = 0;
    }
  }
}

// ---------------------------------------------------------------------------
// Global-memory kernel (batch 5..16): one 16-row tile per CTA of 8 warps,
// weights and activations read straight from global memory.
// ---------------------------------------------------------------------------
template <int QT, int NMG, int EPI>
__global__ void __launch_bounds__(256) k_qmv_reg(const uint8_t* __restrict__ W, int nblk,
                                                 int64_t rows, const uint8_t* __restrict__ xprep,
                                                 int B, float* __restrict__ y, TpArgs tpa) {
  constexpr int TBB = QtInfo<QT>::TBB, QPU = QtInfo<QT>::QPU;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, t = lane & 3;
  const int nunit = (nblk + QPU - 1) / QPU;
  const uint8_t* tile = W + (int64_t)blockIdx.x * nblk * TBB;
  int LW[NMG];
#pragma unroll
  for (int mg = 0; mg < NMG; mg++) LW[mg] = 8 * min(4, B - 4 * mg);
  float tg[NMG], tg8[NMG];
#pragma unroll
  for (int mg = 0; mg < NMG; mg++) tg[mg] = tg8[mg] = 0.f;
  pdl_launch();  // dependents may start their independent prologue now
  pdl_wait();
  for (int u = warp; u < nunit; u += QMV_WARPS) {
    GlobLd ld[NMG];
#pragma unroll
    for (int mg = 0; mg < NMG; mg++) {
      const uint8_t* xu = xprep + xprep_off(mg, nunit, u, LW[mg]);
      ld[mg].w = tile + (int64_t)u * QPU * TBB;
      ld[mg].xf = xu + lane * 16;
      ld[mg].xs = xu + 8 * LW[mg] * 16 + lane * 4;
      ld[mg].xi = xu + 132 * LW[mg] + 4 * t;
      ld[mg].fstride = LW[mg] * 16;
      ld[mg].on = lane < LW[mg];
      ld[mg].oni = 8 * t < LW[mg];
    }
    if (QT == SI_Q4_K) unit_q4k<NMG>(ld, lane, tg, tg8);
    else if (QT == SI_Q6_K) unit_q6k<NMG>(ld, lane, tg, tg8);
    else unit_q80<NMG>(ld, lane, min(QPU, nblk - u * QPU), tg, tg8);
  }
  qmv_epilogue<NMG, EPI>(tg, tg8, B, rows, y, (int)blockIdx.x, tpa);
}

cudaLaunchConfig_t make_cfg(cudaStream_t s, dim3 grid, dim3 block, size_t smem, bool pdl,
                            cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cfg;
}

constexpr int WARP_SMEM_MAX = 220 * 1024;

struct ScratchCap {
  QmvScratch scr;
  size_t split_bytes;
  int64_t count_n;
};

template <int QT, int EPI, int B, int NW, int NS>
int launch_warp_cfg(cudaStream_t s, const si_weight* w, const uint8_t* xprep, float* y,
                    const ScratchCap& scr_cap, int sms, bool pdl) {
  using Cfg = WarpCfg<QT, B, NW, NS>;
  static_assert(Cfg::SMEM <= WARP_SMEM_MAX, "ring too large");
  static DeviceOnce attr_set;
  int dev = 0;
  SI_CUDA(cudaGetDevice(&dev));
  if (!attr_set.done(dev)) {
    SI_CUDA(cudaFuncSetAttribute(k_qmv_warp<QT, EPI, B, NW, NS>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM));
    attr_set.mark(dev);
  }
  const int64_t nunit = (w->nblk + Cfg::QPU - 1) / Cfg::QPU;
  const int64_t units = w->tiles * nunit;
  if (units * sms >= (int64_t)1 << 31)
    SI_FAIL(SI_ERR_UNSUPPORTED, "qmatvec: %lld x %lld is too large for one launch", (long long)w->rows,
            (long long)w->cols);
  // Tile mode (whole row tiles per CTA, no partial sums between CTAs) unless
  // one tile of imbalance costs more than the ~3 us cross-CTA combine; in
  // even-share mode every warp gets a non-empty range (grid * NW <= units).
  const double sm_bytes_us = 6.5e6 / sms;  // bytes per microsecond per SM
  const double ubytes = (double)Cfg::TBB * Cfg::QPU;
  const int64_t g_tile = std::min<int64_t>(w->tiles, sms);
  const double t_tile = (double)((w->tiles + g_tile - 1) / g_tile) * nunit * ubytes / sm_bytes_us;
  const int64_t g_even = qmv_warp_grid(units, NW, sms);
  const double t_even = (double)units * ubytes / (sm_bytes_us * g_even) + 3.0;
  const int tile_mode = t_tile <= t_even ? 1 : 0;
  const int64_t grid = tile_mode ? g_tile : g_even;
  QmvScratch scr = scr_cap.scr;
  scr.maxc = 0;
  if (!tile_mode) {
    const int64_t minr = units / (grid * NW);
    scr.maxc = (int)((nunit - 1 + minr - 1) / minr + 1);
    if ((size_t)w->tiles * scr.maxc * 64 * 4 > scr_cap.split_bytes || w->tiles > scr_cap.count_n)
      SI_FAIL(SI_ERR_INVALID, "qmatvec: scratch too small (need %lld tiles x %d slots)", (long long)w->tiles,
              scr.maxc);
  }
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = make_cfg(s, dim3((unsigned)grid), dim3(NW * 32), Cfg::SMEM, pdl, attr);
  SI_CUDA(cudaLaunchKernelEx(&cfg, k_qmv_warp<QT, EPI, B, NW, NS>, (const uint8_t*)w->dev, (int)w->nblk, w->rows,
                             (int)w->tiles, tile_mode, xprep, y, scr));
  return SI_OK;
}

// 16 warps with the deepest ring (<= 4) that fits, else 8 warps.
template <int QT, int EPI, int B>
int launch_warp(cudaStream_t s, const si_weight* w, const uint8_t* xprep, float* y,
                const ScratchCap& scr, int sms, bool pdl) {
  if constexpr (WarpCfg<QT, B, 16, 4>::SMEM <= WARP_SMEM_MAX)
    return launch_warp_cfg<QT, EPI, B, 16, 4>(s, w, xprep, y, scr, sms, pdl);
  else if constexpr (WarpCfg<QT, B, 16, 3>::SMEM <= WARP_SMEM_MAX)
    return launch_warp_cfg<QT, EPI, B, 16, 3>(s, w, xprep, y, scr, sms, pdl);
  else if constexpr (WarpCfg<QT, B, 16, 2>::SMEM <= WARP_SMEM_MAX)
    return launch_warp_cfg<QT, EPI, B, 16, 2>(s, w, xprep, y, scr, sms, pdl);
  else
    return launch_warp_cfg<QT, EPI, B, 8, 2>(s, w, xprep, y, scr, sms, pdl);
}

template <int QT, int NMG, int EPI>
int launch_reg(cudaStream_t s, const si_weight* w, const uint8_t* xprep, int B, float* y, const TpArgs& tpa,
               bool pdl) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = make_cfg(s, dim3((unsigned)w->tiles), dim3(256), 0, pdl, attr);
  SI_CUDA(cudaLaunchKernelEx(&cfg, k_qmv_reg<QT, NMG, EPI>, (const uint8_t*)w->dev, (int)w->nblk,
                             w->rows, xprep, B, y, tpa));
  return SI_OK;
}

// Batch-1 Q4_K launch; returns -1 when the shape does not suit k_qmv1 (odd
// number of column units, too few unit pairs, or activations too large to
// keep resident in shared memory).
template <int EPI, int NW>
int launch_q1_nw(cudaStream_t s, const si_weight* w, const uint8_t* xprep, float* y, const ScratchCap& scr, int sms,
                 bool pdl, int pmode, const float* xf, const float* nw, float eps) {
  constexpr int NS = 2;
  const int64_t nunit = w->nblk;
  const int64_t P = w->tiles * nunit / 2;
  // the fused RmsNorm holds K <= NW * 512 in registers, read 16 bytes at a time
  if ((pmode == Q1_RMSNORM || pmode == Q1_RMSNORM_TP) &&
      (nunit * 256 > NW * 128 * 4 || (((uintptr_t)xf | (uintptr_t)nw) & 15)))
    return -1;
  // the fused SiLU * up keeps at most 4 units per warp of 16 in registers
  if (pmode == Q1_SILU && (nunit > Q1_SILU_MAX_UNITS * NW / 16 || (((uintptr_t)xf | (uintptr_t)nw) & 15))) return -1;
  const size_t smem = Q1Cfg::smem(NW, NS, (int)nunit, pmode);
  if ((nunit & 1) || P < NW || smem > 227 * 1024 || w->tiles * nunit >= (1 << 24)) return -1;
  static DeviceOnce attr_set, attr_set_tp;
  int dev = 0;
  SI_CUDA(cudaGetDevice(&dev));
  DeviceOnce& once = pmode == Q1_RMSNORM_TP ? attr_set_tp : attr_set;
  if (!once.done(dev)) {
    SI_CUDA(cudaFuncSetAttribute(pmode == Q1_RMSNORM_TP ? k_qmv1<EPI, NW, NS, true> : k_qmv1<EPI, NW, NS, false>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
    once.mark(dev);
  }
  // Tile mode gives every CTA whole row tiles: no partial sums cross CTAs,
  // at the price of up to one tile of imbalance.  Even-share mode balances
  // the pairs exactly but combines the tiles cut between CTAs through global
  // memory (a fence and a counter round trip, ~3 us).  Pick the shorter
  // estimate, streaming at an equal share of the HBM bandwidth per SM.
  const int64_t tiles = w->tiles, npt = nunit / 2;
  const double sm_bytes_us = 6.5e6 / sms;  // bytes per microsecond per SM
  const int64_t g_tile = std::min<int64_t>(tiles, sms);
  const double t_tile = (double)((tiles + g_tile - 1) / g_tile) * nunit * Q1Cfg::TBB / sm_bytes_us;
  const int64_t g_even = std::min<int64_t>(P / NW, sms);
  const double t_even = (double)tiles * nunit * Q1Cfg::TBB / (sm_bytes_us * g_even) + 3.0;
  const int tile_mode = t_tile <= t_even ? 1 : 0;
  const int64_t grid = tile_mode ? g_tile : g_even;
  QmvScratch q = scr.scr;
  q.maxc = 0;
  if (!tile_mode) {
    const int64_t minr = P / (grid * NW);
    q.maxc = (int)((npt - 1 + minr - 1) / minr + 1);
    if ((size_t)tiles * q.maxc * 64 * 4 > scr.split_bytes || tiles > scr.count_n) return -1;
  }
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = make_cfg(s, dim3((unsigned)grid), dim3(NW * 32), smem, pdl, attr);
  SI_CUDA(cudaLaunchKernelEx(&cfg, pmode == Q1_RMSNORM_TP ? k_qmv1<EPI, NW, NS, true> : k_qmv1<EPI, NW, NS, false>,
                             (const uint8_t*)w->dev, (int)nunit, w->rows, (int)tiles,
                             tile_mode, pmode, xprep, xf, nw, eps, y, q));
  return SI_OK;
}

// 16 warps per CTA (one CTA fills an SM), or 8 (half the registers and the
// shared-memory ring, so a CTA of the next kernel can share the SM).
template <int EPI>
int launch_q1(cudaStream_t s, const si_weight* w, const uint8_t* xprep, float* y, const ScratchCap& scr, int sms,
              bool pdl, int pmode = Q1_PREPARED, const float* xf = nullptr, const float* nw = nullptr,
              float eps = 0.f) {
  if (scr.scr.q1w == 8) return launch_q1_nw<EPI, 8>(s, w, xprep, y, scr, sms, pdl, pmode, xf, nw, eps);
  return launch_q1_nw<EPI, 16>(s, w, xprep, y, scr, sms, pdl, pmode, xf, nw, eps);
}

template <int QT, int EPI>
int dispatch_b(cudaStream_t s, const si_weight* w, const uint8_t* xprep, int B, float* y,
               const ScratchCap& scr, int sms, bool pdl) {
  const int64_t units = w->tiles * ((w->nblk + QtInfo<QT>::QPU - 1) / QtInfo<QT>::QPU);
  if (units < 16) B = B <= 4 ? -B : B;  // too small to stream: one CTA per tile
  if constexpr (QT == SI_Q4_K) {
    if (B == 1) {
      const int r = launch_q1<EPI>(s, w, xprep, y, scr, sms, pdl);
      if (r >= 0) return r;
    }
  }
  switch (B) {
    case 1: return launch_warp<QT, EPI, 1>(s, w, xprep, y, scr, sms, pdl);
    case 2: return launch_warp<QT, EPI, 2>(s, w, xprep, y, scr, sms, pdl);
    case 3: return launch_warp<QT, EPI, 3>(s, w, xprep, y, scr, sms, pdl);
    case 4: return launch_warp<QT, EPI, 4>(s, w, xprep, y, scr, sms, pdl);
    default: break;
  }
  if (B < 0) return launch_reg<QT, 1, EPI>(s, w, xprep, -B, y, scr.scr.tp, pdl);
  switch ((B + 3) / 4) {
    case 2: return launch_reg<QT, 2, EPI>(s, w, xprep, B, y, scr.scr.tp, pdl);
    case 3: return launch_reg<QT, 3, EPI>(s, w, xprep, B, y, scr.scr.tp, pdl);
    case 4: return launch_reg<QT, 4, EPI>(s, w, xprep, B, y, scr.scr.tp, pdl);
    default: SI_FAIL(SI_ERR_INVALID, "qmatvec: batch %d outside 1..16", B);
  }
}

template <int EPI>
int dispatch_qt(cudaStream_t s, const si_weight* w, const uint8_t* xprep, int B, float* y,
                const ScratchCap& scr, int sms, bool pdl) {
  switch (w->qtype) {
    case SI_Q4_K: return dispatch_b<SI_Q4_K, EPI>(s, w, xprep, B, y, scr, sms, pdl);
    case SI_Q6_K: return dispatch_b<SI_Q6_K, EPI>(s, w, xprep, B, y, scr, sms, pdl);
    case SI_Q8_0: return dispatch_b<SI_Q8_0, EPI>(s, w, xprep, B, y, scr, sms, pdl);
    default: SI_FAIL(SI_ERR_UNSUPPORTED, "qmatvec: unsupported quant type %d", w->qtype);
  }
}

}  // namespace

int launch_prep(cudaStream_t s, const float* x, int ldx, const float* x2, const float* norm_w,
                float eps, int mode, int K, int B, float* xout, uint8_t* xprep, bool pdl, const PrepTp* tpp) {
  if (K <= 0 || (K & 31)) SI_FAIL(SI_ERR_INVALID, "prep: K=%d must be a positive multiple of 32", K);
  if (K > SI_MAX_K) SI_FAIL(SI_ERR_INVALID, "prep: K=%d above the supported maximum %d", K, SI_MAX_K);
  if (B < 1 || B > SI_MAX_BATCH) SI_FAIL(SI_ERR_INVALID, "prep: batch %d outside 1..%d", B, SI_MAX_BATCH);
  if (mode == SI_PREP_ATTN_MERGE && (ldx < 1 || ldx > SI_ATTN_MAX_SPLITS || K % 128))
    SI_FAIL(SI_ERR_INVALID, "prep: %d attention splits / K=%d", ldx, K);
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = make_cfg(s, dim3(xprep_units(K), B), dim3(256), 0, pdl, attr);
  if (mode == SI_PREP_RMSNORM_TP && (!tpp || !xout)) SI_FAIL(SI_ERR_INVALID, "prep: tensor-parallel mode without peers");
  SI_CUDA(cudaLaunchKernelEx(&cfg, k_prep, x, ldx, x2, norm_w, eps, mode, K, B, xout, xprep,
                             tpp ? *tpp : PrepTp{}));
  return SI_OK;
}

// y (op)= W RmsNorm(x) nw for one row x: the batch-1 Q4_K kernel normalises
// and prepares x itself; other weights go through k_prep into xprep first.
int launch_qmv_rms(cudaStream_t s, const si_weight* w, const float* x, const float* nw, float eps, float* y,
                   int epi, const QmvBuffers& qb, uint8_t* xprep, bool pdl) {
  if (w->qtype == SI_Q4_K && (epi == SI_EPI_STORE || epi == SI_EPI_ADD)) {
    const ScratchCap scr{QmvScratch{qb.split, qb.count, qb.err, 0, qb.tp, qb.pf, qb.ring_mode, qb.q1w}, qb.split_bytes, qb.count_n};
    const int r = epi == SI_EPI_ADD
                      ? launch_q1<SI_EPI_ADD>(s, w, nullptr, y, scr, qb.sms, pdl, Q1_RMSNORM, x, nw, eps)
                      : launch_q1<SI_EPI_STORE>(s, w, nullptr, y, scr, qb.sms, pdl, Q1_RMSNORM, x, nw, eps);
    if (r >= 0) return r;
  }
  SI_TRY(launch_prep(s, x, (int)w->cols, nullptr, nw, eps, SI_PREP_RMSNORM, (int)w->cols, 1, nullptr, xprep, pdl));
  return launch_qmv(s, w, xprep, 1, y, epi, qb, pdl);
}

// y = W RmsNorm(xres + sum over ranks of the partial sums) nw for one row
// (tensor parallel, batch 1), with the new residual written to xout: inside
// the batch-1 Q4_K kernel where it applies (returns -1 otherwise).
int launch_qmv_rms_tp(cudaStream_t s, const si_weight* w, const float* xres, float* xout, const float* nw, float eps,
                      float* y, const QmvBuffers& qb, const PrepTp& pt, bool pdl) {
  if (w->qtype != SI_Q4_K || !pt.comm || !pt.epoch || pt.tp < 1 || pt.tp > SI_TP_MAX || ((uintptr_t)xout & 15))
    return -1;
  ScratchCap scr{QmvScratch{qb.split, qb.count, qb.err, 0, qb.tp, qb.pf, qb.ring_mode, qb.q1w}, qb.split_bytes, qb.count_n};
  scr.scr.ptp = pt;
  scr.scr.xout = xout;
  return launch_q1<SI_EPI_STORE>(s, w, nullptr, y, scr, qb.sms, pdl, Q1_RMSNORM_TP, xres, nw, eps);
}

// y (op)= W (SiLU(gate) * up) for one row (batch 1): the batch-1 Q4_K kernel
// computes and prepares its input itself; otherwise k_prep does it first.
int launch_qmv_silu(cudaStream_t s, const si_weight* w, const float* gate, const float* up, float* y, int epi,
                    const QmvBuffers& qb, uint8_t* xprep, bool pdl) {
  if (w->qtype == SI_Q4_K) {
    const ScratchCap scr{QmvScratch{qb.split, qb.count, qb.err, 0, qb.tp, qb.pf, qb.ring_mode, qb.q1w}, qb.split_bytes, qb.count_n};
    int r = -1;
    if (epi == SI_EPI_ADD) r = launch_q1<SI_EPI_ADD>(s, w, nullptr, y, scr, qb.sms, pdl, Q1_SILU, gate, up);
    else if (epi == SI_EPI_STORE) r = launch_q1<SI_EPI_STORE>(s, w, nullptr, y, scr, qb.sms, pdl, Q1_SILU, gate, up);
    else if (epi == SI_EPI_TP) r = launch_q1<SI_EPI_TP>(s, w, nullptr, y, scr, qb.sms, pdl, Q1_SILU, gate, up);
    if (r >= 0) return r;
  }
  const int K = (int)w->cols;
  SI_TRY(launch_prep(s, gate, K, up, nullptr, 0.f, SI_PREP_SILU_MUL, K, 1, nullptr, xprep, pdl));
  return launch_qmv(s, w, xprep, 1, y, epi, qb, pdl);
}

int launch_qmv(cudaStream_t s, const si_weight* w, const uint8_t* xprep, int B, float* y, int epi,
               const QmvBuffers& qb, bool pdl) {
  const ScratchCap scr{QmvScratch{qb.split, qb.count, qb.err, 0, qb.tp, qb.pf, qb.ring_mode, qb.q1w}, qb.split_bytes, qb.count_n};
  if (epi == SI_EPI_TP && (qb.tp.tp < 1 || !qb.tp.peers || !qb.tp.epoch))
    SI_FAIL(SI_ERR_INVALID, "qmatvec: tensor-parallel epilogue without peers");
  if (B > 4 && (w->qtype == SI_Q4_K || w->qtype == SI_Q6_K) && qmv_wide_enabled()) {  // batch 5..16
    const int r = launch_qmv_wide(s, w, xprep, B, y, epi, qb, pdl);
    if (r >= 0) return r;
  }
  if (epi == SI_EPI_ADD) return dispatch_qt<SI_EPI_ADD>(s, w, xprep, B, y, scr, qb.sms, pdl);
  if (epi == SI_EPI_TP) {
    if (qb.tp.tp < 1 || !qb.tp.peers || !qb.tp.epoch) SI_FAIL(SI_ERR_INVALID, "qmatvec: tensor-parallel epilogue without peers");
    return dispatch_qt<SI_EPI_TP>(s, w, xprep, B, y, scr, qb.sms, pdl);
  }
  return dispatch_qt<SI_EPI_STORE>(s, w, xprep, B, y, scr, qb.sms, pdl);
}

}  // namespace si
