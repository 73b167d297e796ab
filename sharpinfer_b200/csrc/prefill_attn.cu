// Prefill attention on the 5th-generation tensor cores: the tiled
// online-softmax algorithm of FlashAttention.Forward
// (src/SharpInfer.Core/Layers/FlashAttention.cs:59-167) for bf16 Q, K, V with
// grouped-query heads and a causal offset.
//
// O[b][h][i] = sum_j softmax_j(Q[b][h][i] . K[b][h/G][j] * scale) V[b][h/G][j]
// over keys j <= i + start_pos (causal) or all keys; a row without a visible
// key is 0 (FlashAttention.cs:155-163).  Accumulation is f32 throughout; Q,
// K, V enter exactly (they are bf16), the probabilities as bf16 hi + lo.
#include <cuda_bf16.h>

#include "common.cuh"
#include "tcgen05.cuh"

namespace si {
namespace {

constexpr int PA_D = 128;  // head dimension

// 2^x by the hardware approximation (relative error ~2^-22; 2^-inf = 0,
// results below 2^-126 flushed to 0), one instruction.
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ---------------------------------------------------------------------------
// tcgen05 flash attention.  One CTA = 128 queries (M) of one head, key tiles
// of 64 (N).  Warp 0: TMA (Q once, K and V^T tiles through a 3-stage ring);
// warp 1: tcgen05.mma issuer; warps 2-9: softmax, two threads per query row
// (TMEM lanes 32 (warp % 4) .. + 31), warps 2-5 on key columns 0-31 and
// output dims 0-63, warps 6-9 on the other halves; the two warps of a row
// quarter exchange their row maxima through shared memory (a 64-thread named
// barrier per pair).  Per key tile j:
//   S_j = Q K_j^T            (M 128, N 64, K 128: 8 MMAs) -> TMEM S[j % 2]
//   softmax: masked row max, p = exp(s - m), running sum, P_j written to
//            shared memory as bf16 hi + lo in the K-major 128-byte-swizzled
//            A-operand layout
//   O += P_hi V_j + P_lo V_j (M 128, N 128, K 64: 8 MMAs), one TMEM accumulator
//   the maximum in use is raised only when the row maximum passes it by
//   more than 8 (base 2); then the softmax threads rescale O in TMEM first.
// S_{j+1} is issued before O_j, so the softmax of tile j overlaps it.  V is
// used transposed (V^T [d][keys], made by k_vt) so that both operands of
// every MMA are K-major.  All waits are bounded.
constexpr int FA_BQ = 128, FA_BK = 64, FA_NST = 3;
constexpr int FA_QB = FA_BQ * 256;  // Q: two 64-dim chunks of [128 rows][128 B]
constexpr int FA_KB = FA_BK * 256;  // K tile: two chunks of [64 keys][128 B]
constexpr int FA_VB = 128 * 128;    // V^T tile: [128 dims][64 keys * 2 B]
constexpr int FA_PB = FA_BQ * 128;  // P (hi or lo): [128 rows][64 keys * 2 B]
constexpr int FA_XCH = 3 * 256 * 4;  // row maxima [2 tiles][2 halves][128] and row sums [2][128]
constexpr int FA_SMEM = 1024 + FA_QB + FA_NST * (FA_KB + FA_VB) + 4 * FA_PB + 256 + FA_XCH;
constexpr int FA_THREADS = 320;  // TMA warp, MMA warp, 8 softmax warps
// kind::f16 instruction descriptors: D f32, A and B bf16 (bits 7, 10) or f16
// (format 0), both K-major
template <bool F16>
struct FaDesc {
  static constexpr uint32_t AB = F16 ? 0u : ((1u << 7) | (1u << 10));
  static constexpr uint32_t S = (1u << 4) | AB | ((64u >> 3) << 17) | ((128u >> 4) << 24);
  static constexpr uint32_t O = (1u << 4) | AB | ((128u >> 3) << 17) | ((128u >> 4) << 24);
};

// One 16-bit operand type for Q, K, V and the probabilities: bf16 (the
// public bf16 entry point) or f16 (the model's f16 KV cache).
template <bool F16>
__device__ __forceinline__ void split_pair(float a0, float a1, uint32_t& hi, uint32_t& lo) {
  if (F16) {
    const __half2 h = __floats2half2_rn(a0, a1);
    const float2 hf = __half22float2(h);
    const __half2 lw = __floats2half2_rn(a0 - hf.x, a1 - hf.y);
    hi = *(const uint32_t*)&h;
    lo = *(const uint32_t*)&lw;
  } else {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a0, a1);
    const float2 hf = __bfloat1622float2(h);
    const __nv_bfloat162 lw = __floats2bfloat162_rn(a0 - hf.x, a1 - hf.y);
    hi = *(const uint32_t*)&h;
    lo = *(const uint32_t*)&lw;
  }
}

template <bool F16>
__global__ void __launch_bounds__(FA_THREADS, 1) k_attn_fa_tc(const __grid_constant__ CUtensorMap tmQ,
                                                       const __grid_constant__ CUtensorMap tmK,
                                                       const __grid_constant__ CUtensorMap tmV, float* __restrict__ O,
                                                       int Hq, int Hkv, int S, int KV, float scale, int causal,
                                                       int start_pos, int* err) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t sQ = base, sK = sQ + FA_QB, sV = sK + FA_NST * FA_KB, sP = sV + FA_NST * FA_VB;
  const uint32_t bars = sP + 4 * FA_PB;
  float* xch = (float*)(smem_raw + (bars + 256 - smem_u32(smem_raw)));  // [3][256] f32
  // barriers: kv_full[NST] kv_empty[NST] s_full[2] s_free[2] p_full[2] o_full[2] (unused slot) q_full, TMEM slot
  const uint32_t kv_full = bars, kv_empty = bars + 8 * FA_NST, s_full = bars + 16 * FA_NST, s_free = s_full + 16,
                 p_full = s_full + 32, o_full = s_full + 48, q_full = s_full + 80,
                 tslot = s_full + 88;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qblk = causal ? (int)gridDim.x - 1 - (int)blockIdx.x : (int)blockIdx.x;  // longest key ranges first
  const int q0 = qblk * FA_BQ, h = blockIdx.y, b = blockIdx.z, hk = h / (Hq / Hkv);
  const int kend = causal ? min(KV, q0 + FA_BQ + start_pos) : KV;
  const int nt = kend > 0 ? (kend + FA_BK - 1) / FA_BK : 0;
  if (threadIdx.x == 0) {
    for (int i = 0; i < FA_NST; i++) {
      mbar_init(kv_full + 8 * i, 1);
      mbar_init(kv_empty + 8 * i, 1);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(s_full + 8 * i, 1);
      mbar_init(s_free + 8 * i, 256);
      mbar_init(p_full + 8 * i, 256);
      mbar_init(o_full + 8 * i, 1);
    }
    mbar_init(q_full, 1);
    mbar_fence_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tslot), "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = lds_u32(tslot);
  bool ok = true;
  if (warp == 0) {
    if (lane == 0) {  // TMA producer
      mbar_arrive_expect_tx(q_full, FA_QB);
      tma_load_3d(sQ, &tmQ, 0, q0, b * Hq + h, q_full);
      tma_load_3d(sQ + FA_QB / 2, &tmQ, 64, q0, b * Hq + h, q_full);
      for (int j = 0; j < nt && ok; j++) {
        const int st = j % FA_NST;
        if (ok && j >= FA_NST && !mbar_wait_bounded(kv_empty + 8 * st, (uint32_t)((j / FA_NST - 1) & 1))) ok = false;
        mbar_arrive_expect_tx(kv_full + 8 * st, FA_KB + FA_VB);
        tma_load_3d(sK + st * FA_KB, &tmK, 0, j * FA_BK, b * Hkv + hk, kv_full + 8 * st);
        tma_load_3d(sK + st * FA_KB + FA_KB / 2, &tmK, 64, j * FA_BK, b * Hkv + hk, kv_full + 8 * st);
        tma_load_3d(sV + st * FA_VB, &tmV, j * FA_BK, 0, b * Hkv + hk, kv_full + 8 * st);
      }
      if (!ok) atomicOr(err, SI_DEVERR_WAIT_TIMEOUT);
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      if (ok && !mbar_wait_bounded(q_full, 0)) ok = false;
      auto issue_s = [&](int j) {
        const int st = j % FA_NST;
        if (ok && !mbar_wait_bounded(kv_full + 8 * st, (uint32_t)((j / FA_NST) & 1))) ok = false;
        if (ok && j >= 2 && !mbar_wait_bounded(s_free + 8 * (j & 1), (uint32_t)((j / 2 - 1) & 1))) ok = false;
        tc_fence_after();
        if (ok) {
#pragma unroll
          for (int c = 0; c < 2; c++)
#pragma unroll
            for (int kk = 0; kk < 4; kk++)
              umma_f16(tmem + 64 * (j & 1), sdesc_k128(sQ + c * (FA_QB / 2)) + 2 * kk,
                       sdesc_k128(sK + st * FA_KB + c * (FA_KB / 2)) + 2 * kk, FaDesc<F16>::S, (c | kk) != 0);
        }
        umma_commit(s_full + 8 * (j & 1));
      };
      if (nt > 0) issue_s(0);
      for (int j = 0; j < nt; j++) {
        if (j + 1 < nt) issue_s(j + 1);
        const int st = j % FA_NST, pb = j & 1;
        if (ok && !mbar_wait_bounded(p_full + 8 * pb, (uint32_t)((j / 2) & 1))) ok = false;
        tc_fence_after();
        if (ok) {  // O accumulates over the tiles in one TMEM buffer
          const uint32_t ph = sP + pb * 2 * FA_PB, vt = sV + st * FA_VB, d = tmem + 128;
#pragma unroll
          for (int kk = 0; kk < 4; kk++)
            umma_f16(d, sdesc_k128(ph) + 2 * kk, sdesc_k128(vt) + 2 * kk, FaDesc<F16>::O, (j | kk) != 0);
#pragma unroll
          for (int kk = 0; kk < 4; kk++)
            umma_f16(d, sdesc_k128(ph + FA_PB) + 2 * kk, sdesc_k128(vt) + 2 * kk, FaDesc<F16>::O, 1);
        }
        umma_commit(o_full + 8 * pb);
        umma_commit(kv_empty + 8 * st);
      }
      if (!ok) atomicOr(err, SI_DEVERR_WAIT_TIMEOUT);
    }
  } else {  // softmax: two threads per query row r of the tile
    const int qq = warp & 3, half = (warp - 2) >> 2, r = 32 * qq + lane, qrow = q0 + r;
    const uint32_t lanes = (uint32_t)(32 * qq) << 16;
    const uint32_t ocol = tmem + lanes + 128 + 64 * half;  // this thread's 64 dims of O
    // Base-2 units: t = s * scale * log2(e), p = 2^(t - m) = e^(s scale - m')
    // with m the maximum in use.  O accumulates in TMEM with that m; it is
    // raised (and O and l rescaled) only when the row maximum exceeds it by
    // more than 8, so p <= 2^8 and most tiles need no rescale.
    float m = -INFINITY, l = 0.f;  // l over this thread's keys
    const float sc2 = scale * 1.4426950408889634f;  // scale * log2(e)
    for (int j = 0; j < nt; j++) {
      const int pb = j & 1;
      if (ok && !mbar_wait_bounded(s_full + 8 * pb, (uint32_t)((j / 2) & 1))) ok = false;
      tc_fence_after();
      float sv[32];
      {
        uint32_t r32[32];
        tmem_ld32(tmem + lanes + 64 * pb + 32 * half, r32);
#pragma unroll
        for (int i = 0; i < 32; i++) sv[i] = __uint_as_float(r32[i]);
      }
      tc_fence_before();
      mbar_arrive(s_free + 8 * pb);
      // mask, row maximum (FlashAttention.cs:206-224, 238-325)
      const int k0 = j * FA_BK + 32 * half;
      const bool full = k0 + 32 <= KV && (!causal || k0 + 31 <= q0 + start_pos);  // no key masked
      float mx = -INFINITY;
      if (full) {
#pragma unroll
        for (int i = 0; i < 32; i++) {
          sv[i] *= sc2;
          mx = fmaxf(mx, sv[i]);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; i++) {
          const int key = k0 + i;
          const float v = (key >= KV || (causal && key > qrow + start_pos)) ? -INFINITY : sv[i] * sc2;
          sv[i] = v;
          mx = fmaxf(mx, v);
        }
      }
      xch[pb * 256 + half * 128 + r] = mx;  // the row maximum needs both halves
      asm volatile("bar.sync %0, 64;" ::"r"(1 + qq) : "memory");  // the two warps of this row quarter
      mx = fmaxf(mx, xch[pb * 256 + (half ^ 1) * 128 + r]);
      if (mx > m + 8.f) {  // raise the maximum in use (both threads of the row decide alike)
        const bool had = m != -INFINITY;
        const float alpha = had ? ex2(m - mx) : 0.f;
        l *= alpha;
        m = mx;
        if (had && j >= 1) {  // O so far (tiles < j) is complete and rescaled in place
          if (ok && !mbar_wait_bounded(o_full + 8 * ((j - 1) & 1), (uint32_t)(((j - 1) / 2) & 1))) ok = false;
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < 2; c++) {
            uint32_t t32[32];
            tmem_ld32(ocol + 32 * c, t32);
#pragma unroll
            for (int i = 0; i < 32; i++) t32[i] = __float_as_uint(__uint_as_float(t32[i]) * alpha);
            tmem_st32(ocol + 32 * c, t32);
          }
          tc_fence_before();
        }
      }
      float ps = 0.f;
      if (m != -INFINITY) {
#pragma unroll
        for (int i = 0; i < 32; i++) {
          const float p = ex2(sv[i] - m);  // 2^-inf = 0 for masked keys; <= 2^8
          sv[i] = p;
          ps += p;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; i++) sv[i] = 0.f;
      }
      l += ps;
      // P_j goes to the buffer P_{j-2} used: wait for that product
      if (ok && j >= 2 && !mbar_wait_bounded(o_full + 8 * pb, (uint32_t)(((j - 2) / 2) & 1))) ok = false;
      {  // P_j as hi + lo (bf16 or f16): row r, chunks of 8 keys, chunk g at (g ^ (r % 8)) * 16 in the 128-byte row
        const uint32_t ph = sP + pb * 2 * FA_PB + r * 128;
#pragma unroll
        for (int gg = 0; gg < 4; gg++) {
          const int g = 4 * half + gg;
          uint32_t hi[4], lo[4];
#pragma unroll
          for (int e = 0; e < 4; e++) {
            split_pair<F16>(sv[8 * gg + 2 * e], sv[8 * gg + 2 * e + 1], hi[e], lo[e]);
          }
          const uint32_t off = (uint32_t)((g ^ (r & 7)) << 4);
          asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(ph + off), "r"(hi[0]), "r"(hi[1]), "r"(hi[2]),
                       "r"(hi[3])
                       : "memory");
          asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(ph + FA_PB + off), "r"(lo[0]), "r"(lo[1]),
                       "r"(lo[2]), "r"(lo[3])
                       : "memory");
        }
      }
      fence_proxy_async_smem();
      mbar_arrive(p_full + 8 * pb);
    }
    xch[512 + half * 128 + r] = l;  // the row sum adds both halves' keys
    asm volatile("bar.sync %0, 64;" ::"r"(1 + qq) : "memory");
    const float lr = l + xch[512 + (half ^ 1) * 128 + r];
    float oacc[64];
    if (nt > 0) {  // O after the last tile's product
      const int jl = nt - 1;
      if (ok && !mbar_wait_bounded(o_full + 8 * (jl & 1), (uint32_t)((jl / 2) & 1))) ok = false;
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < 2; c++) {
        uint32_t t32[32];
        tmem_ld32(ocol + 32 * c, t32);
#pragma unroll
        for (int i = 0; i < 32; i++) oacc[32 * c + i] = __uint_as_float(t32[i]);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 64; i++) oacc[i] = 0.f;
    }
    if (!ok && lane == 0) atomicOr(err, SI_DEVERR_WAIT_TIMEOUT);
    if (qrow < S) {  // a row without a visible key is 0 (FlashAttention.cs:155-163)
      const float inv = lr > 0.f ? 1.0f / lr : 0.f;
      float4* orow = (float4*)(O + (((int64_t)b * Hq + h) * S + qrow) * PA_D + 64 * half);
#pragma unroll
      for (int i = 0; i < 16; i++)
        orow[i] = make_float4(oacc[4 * i] * inv, oacc[4 * i + 1] * inv, oacc[4 * i + 2] * inv, oacc[4 * i + 3] * inv);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
  }
}

// V [bh][kv][128] -> V^T [bh][128][kvp] (keys >= kv zero), 32 x 32 tiles.
__global__ void k_vt(const uint16_t* __restrict__ V, uint16_t* __restrict__ Vt, int kv, int kvp) {
  __shared__ uint16_t t[32][34];
  const int bh = blockIdx.z, k0 = blockIdx.x * 32, d0 = blockIdx.y * 32;
  const uint16_t* src = V + (int64_t)bh * kv * PA_D;
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int k = k0 + i;
    t[i][threadIdx.x] = k < kv ? src[(int64_t)k * PA_D + d0 + threadIdx.x] : (uint16_t)0;
  }
  __syncthreads();
  uint16_t* dst = Vt + (int64_t)bh * PA_D * kvp;
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int k = k0 + threadIdx.x;
    if (k < kvp) dst[(int64_t)(d0 + i) * kvp + k] = t[threadIdx.x][i];
  }
}

// 3D 16-bit tensor [n2][n1][n0] (n0 contiguous), box [b2 = 1][b1][64], 128-byte swizzle.
int make_tmap3(CUtensorMap* tm, const void* ptr, int64_t n0, int64_t n1, int64_t n2, int b1, bool f16) {
  auto fn = encode_fn();
  if (!fn) SI_FAIL(SI_ERR_CUDA, "si_attn_prefill: cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[3] = {(cuuint64_t)n0, (cuuint64_t)n1, (cuuint64_t)n2};
  const cuuint64_t strides[2] = {(cuuint64_t)n0 * 2, (cuuint64_t)n0 * n1 * 2};
  const cuuint32_t box[3] = {64, (cuuint32_t)b1, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(tm, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                        const_cast<void*>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) SI_FAIL(SI_ERR_CUDA, "si_attn_prefill: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return SI_OK;
}

}  // namespace

// Prefill attention for q [batch][heads][seq][128], k, v [batch][kv_heads][kv][128]
// (16-bit: bf16, or f16 when f16 is set) into o f32 [batch][heads][seq][128],
// asynchronous on the context stream; the checks of si_attn_prefill apply.
int launch_attn_prefill(si_ctx* c, const uint16_t* q, const uint16_t* k, const uint16_t* v, float* o, int batch,
                        int heads, int kv_heads, int seq, int kv, float scale, int causal, int start_pos, bool f16) {
  if (kv > 0) {  // tensor cores (tcgen05): V transposed into scratch, Q/K/V^T through TMA
    const int kvp = (kv + 7) & ~7;  // 16-byte rows of V^T
    SI_TRY(ensure(c->stage[3], (size_t)batch * kv_heads * PA_D * kvp * 2));
    uint16_t* vt = (uint16_t*)c->stage[3].ptr;
    k_vt<<<dim3((unsigned)((kvp + 31) / 32), PA_D / 32, (unsigned)(batch * kv_heads)), dim3(32, 8), 0, c->stream>>>(
        v, vt, kv, kvp);
    SI_CUDA(cudaGetLastError());
    CUtensorMap tq, tk, tv;
    SI_TRY(make_tmap3(&tq, q, PA_D, seq, (int64_t)batch * heads, FA_BQ, f16));
    SI_TRY(make_tmap3(&tk, k, PA_D, kv, (int64_t)batch * kv_heads, FA_BK, f16));
    SI_TRY(make_tmap3(&tv, vt, kvp, PA_D, (int64_t)batch * kv_heads, PA_D, f16));
    static DeviceOnce fa_attr[2];
    if (!fa_attr[f16].done(c->device)) {
      if (f16) SI_CUDA(cudaFuncSetAttribute(k_attn_fa_tc<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, FA_SMEM));
      else SI_CUDA(cudaFuncSetAttribute(k_attn_fa_tc<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, FA_SMEM));
      fa_attr[f16].mark(c->device);
    }
    dim3 grid((unsigned)((seq + FA_BQ - 1) / FA_BQ), (unsigned)heads, (unsigned)batch);
    if (f16)
      k_attn_fa_tc<true><<<grid, FA_THREADS, FA_SMEM, c->stream>>>(tq, tk, tv, o, heads, kv_heads, seq, kv, scale,
                                                                   causal, start_pos, c->dev_err);
    else
      k_attn_fa_tc<false><<<grid, FA_THREADS, FA_SMEM, c->stream>>>(tq, tk, tv, o, heads, kv_heads, seq, kv, scale,
                                                                    causal, start_pos, c->dev_err);
    SI_CUDA(cudaGetLastError());
    return SI_OK;
  }
  // no keys: every row sees none and is 0 (FlashAttention.cs:155-163)
  SI_CUDA(cudaMemsetAsync(o, 0, (size_t)batch * heads * seq * PA_D * 4, c->stream));
  SI_CUDA(cudaGetLastError());
  return SI_OK;
}

}  // namespace si

using namespace si;

extern "C" SI_EXPORT int si_attn_prefill(si_ctx* c, const uint16_t* q, const uint16_t* k, const uint16_t* v, float* o,
                                         int batch, int heads, int kv_heads, int seq, int kv, int head_dim,
                                         float scale, int causal, int start_pos) {
  clear_error();
  if (!c || !q || !o || (kv > 0 && (!k || !v))) SI_FAIL(SI_ERR_INVALID, "si_attn_prefill: NULL argument");
  if (head_dim != PA_D) SI_FAIL(SI_ERR_UNSUPPORTED, "si_attn_prefill: head_dim %d (this build supports 128)", head_dim);
  if (batch < 1 || heads < 1 || kv_heads < 1 || heads % kv_heads || seq < 1 || kv < 0)
    SI_FAIL(SI_ERR_INVALID, "si_attn_prefill: bad shape");
  if (batch > 65535 || heads > 65535) SI_FAIL(SI_ERR_UNSUPPORTED, "si_attn_prefill: batch/heads above 65535");
  if (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)o) & 15)
    SI_FAIL(SI_ERR_INVALID, "si_attn_prefill: buffers must be 16-byte aligned");
  SI_TRY(bind_device(c));
  return launch_attn_prefill(c, q, k, v, o, batch, heads, kv_heads, seq, kv, scale, causal, start_pos, false);
}
