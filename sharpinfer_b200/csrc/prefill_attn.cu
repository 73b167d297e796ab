// Prefill attention on the tensor cores: the tiled online-softmax algorithm of
// FlashAttention.Forward (src/SharpInfer.Core/Layers/FlashAttention.cs:59-167)
// for bf16 Q, K, V with grouped-query heads and a causal offset.
//
// O[b][h][i] = sum_j softmax_j(Q[b][h][i] . K[b][h/G][j] * scale) V[b][h/G][j]
// over keys j <= i + start_pos (causal) or all keys; a row without a visible
// key is 0 (FlashAttention.cs:155-163).
//
// One CTA = 64 queries of one head (4 warps x 16 rows).  Key/value tiles of 64
// positions are staged in shared memory by cp.async (16-byte chunks XOR
// swizzled by row, so ldmatrix is conflict free) with double buffering.
//  * S = Q K^T: mma.m16n8k16 bf16 -> f32, Q A-fragments kept in registers,
//    K B-fragments straight from ldmatrix;
//  * online softmax per row in registers (running max, sum);
//  * O += P V: P is split into bf16 hi + lo (P = hi + lo to ~16 bits), two
//    MMAs per step, V B-fragments from ldmatrix.trans.
// Accumulation is f32 throughout; Q, K, V enter exactly (they are bf16).
//
// On sm_100 the attention runs on the 5th-generation tensor cores instead
// (k_attn_fa_tc below): S = Q K^T and the P V of each key tile accumulate in
// tensor memory, the softmax warps keep O in registers.  The mma.sync
// kernel above serves shapes the tensor-map path does not take.
#include <cuda_bf16.h>

#include "common.cuh"
#include "tcgen05.cuh"

namespace si {
namespace {

constexpr int PA_D = 128;       // head dimension
constexpr int PA_BQ = 64;       // queries per CTA
constexpr int PA_BK = 64;       // keys per tile
constexpr int PA_ROW = PA_D * 2;  // bytes per row (256)
constexpr int PA_TILE = PA_BK * PA_ROW;  // 16 KB

__device__ __forceinline__ uint32_t swz(int row, int chunk) { return (uint32_t)(row * PA_ROW + ((chunk ^ (row & 7)) << 4)); }

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;  // zero-fill rows past the end
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldsm4(uint32_t a, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(a));
}
__device__ __forceinline__ void ldsm4t(uint32_t a, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(a));
}
__device__ __forceinline__ void mma_bf16(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t bf2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *(const uint32_t*)&v;
}
__device__ __forceinline__ float bf_round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// Copy rows [r0, r0 + 64) of a [rows][128] bf16 matrix into a swizzled tile
// (rows >= nrows are zero-filled); 128 threads, 8 chunks each.
__device__ __forceinline__ void load_tile(uint32_t tile, const __nv_bfloat16* src, int r0, int nrows, int tid) {
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const int idx = tid + 128 * i, row = idx >> 4, chunk = idx & 15;
    const bool v = r0 + row < nrows;
    const __nv_bfloat16* p = src + (int64_t)(v ? r0 + row : 0) * PA_D + chunk * 8;
    cp_async16(tile + swz(row, chunk), p, v);
  }
}

__global__ void __launch_bounds__(128) k_attn_prefill(const __nv_bfloat16* __restrict__ Q,
                                                      const __nv_bfloat16* __restrict__ K,
                                                      const __nv_bfloat16* __restrict__ V, float* __restrict__ O,
                                                      int Hq, int Hkv, int S, int KV, float scale, int causal,
                                                      int start_pos) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int q0 = blockIdx.x * PA_BQ, h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (Hq / Hkv);
  const __nv_bfloat16* qb = Q + ((int64_t)b * Hq + h) * S * PA_D;
  const __nv_bfloat16* kb = K + ((int64_t)b * Hkv + hk) * KV * PA_D;
  const __nv_bfloat16* vb = V + ((int64_t)b * Hkv + hk) * KV * PA_D;
  const uint32_t sq = smem_u32(smem);
  const uint32_t sk[2] = {sq + PA_TILE, sq + 2 * PA_TILE};
  const uint32_t sv[2] = {sq + 3 * PA_TILE, sq + 4 * PA_TILE};

  // keys this CTA can see: j <= q0 + 63 + start_pos (causal)
  int kend = KV;
  if (causal) kend = min(KV, q0 + PA_BQ + start_pos);
  const int ntiles = kend > 0 ? (kend + PA_BK - 1) / PA_BK : 0;

  load_tile(sq, qb, q0, S, tid);
  if (ntiles > 0) {
    load_tile(sk[0], kb, 0, KV, tid);
    load_tile(sv[0], vb, 0, KV, tid);
  }
  cp_commit();

  // this warp's 16 query rows: g and g+8 of rows q0 + 16 warp
  const int qr0 = q0 + 16 * warp + g, qr1 = qr0 + 8;
  float o[16][4];  // 128 dims = 16 n-tiles of 8; per n-tile: rows g (0,1), g+8 (2,3), cols 2t, 2t+1
#pragma unroll
  for (int n = 0; n < 16; n++) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  uint32_t qa[8][4];  // Q A-fragments for 8 k-steps of 16 dims

  for (int it = 0; it < ntiles; it++) {
    const int cur = it & 1;
    if (it + 1 < ntiles) {  // prefetch the next tile
      load_tile(sk[cur ^ 1], kb, (it + 1) * PA_BK, KV, tid);
      load_tile(sv[cur ^ 1], vb, (it + 1) * PA_BK, KV, tid);
    }
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    if (it == 0) {
#pragma unroll
      for (int ks = 0; ks < 8; ks++) {  // A (16 rows x 16 dims): matrices (rows 0-7|8-15) x (dims 0-7|8-15)
        const int m = lane >> 3, r = 16 * warp + (lane & 7) + 8 * (m & 1), c = 2 * ks + (m >> 1);
        ldsm4(sq + swz(r, c), qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3]);
      }
    }
    // ---- S = Q K^T for 64 keys: 8 n-tiles of 8 keys ----
    float s[8][4];
#pragma unroll
    for (int n = 0; n < 8; n++) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ks++) {
#pragma unroll
      for (int np = 0; np < 4; np++) {  // two n-tiles (16 keys) per ldmatrix.x4
        // B (16 dims x 8 keys) for keys 16np..+7 and +8..+15: matrices (keys 0-7|8-15) x (dims 0-7|8-15)
        const int m = lane >> 3, r = 16 * np + (lane & 7) + 8 * (m >> 1), c = 2 * ks + (m & 1);
        uint32_t b0, b1, b2, b3;
        ldsm4(sk[cur] + swz(r, c), b0, b1, b2, b3);
        mma_bf16(s[2 * np], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b0, b1);
        mma_bf16(s[2 * np + 1], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b2, b3);
      }
    }
    // ---- mask, online softmax (FlashAttention.cs:238-325) ----
    const int k0 = it * PA_BK;
    float bm0 = -INFINITY, bm1 = -INFINITY;
#pragma unroll
    for (int n = 0; n < 8; n++)
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const int key = k0 + 8 * n + 2 * t + (e & 1);
        const int qr = e < 2 ? qr0 : qr1;
        float v = s[n][e] * scale;
        if (key >= KV || (causal && key > qr + start_pos)) v = -INFINITY;
        s[n][e] = v;
        if (e < 2) bm0 = fmaxf(bm0, v);
        else bm1 = fmaxf(bm1, v);
      }
    bm0 = fmaxf(bm0, __shfl_xor_sync(0xFFFFFFFFu, bm0, 1));
    bm0 = fmaxf(bm0, __shfl_xor_sync(0xFFFFFFFFu, bm0, 2));
    bm1 = fmaxf(bm1, __shfl_xor_sync(0xFFFFFFFFu, bm1, 1));
    bm1 = fmaxf(bm1, __shfl_xor_sync(0xFFFFFFFFu, bm1, 2));
    const float nm0 = fmaxf(m0, bm0), nm1 = fmaxf(m1, bm1);
    const float r0 = nm0 == -INFINITY ? 1.f : expf(m0 - nm0), r1 = nm1 == -INFINITY ? 1.f : expf(m1 - nm1);
    m0 = nm0;
    m1 = nm1;
    float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
    for (int n = 0; n < 8; n++)
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const float mm = e < 2 ? m0 : m1;
        const float p = s[n][e] == -INFINITY ? 0.f : expf(s[n][e] - mm);
        s[n][e] = p;
        if (e < 2) ps0 += p;
        else ps1 += p;
      }
    ps0 += __shfl_xor_sync(0xFFFFFFFFu, ps0, 1);
    ps0 += __shfl_xor_sync(0xFFFFFFFFu, ps0, 2);
    ps1 += __shfl_xor_sync(0xFFFFFFFFu, ps1, 1);
    ps1 += __shfl_xor_sync(0xFFFFFFFFu, ps1, 2);
    l0 = l0 * r0 + ps0;
    l1 = l1 * r1 + ps1;
#pragma unroll
    for (int n = 0; n < 16; n++) {
      o[n][0] *= r0;
      o[n][1] *= r0;
      o[n][2] *= r1;
      o[n][3] *= r1;
    }
    // ---- O += P V: k-steps of 16 keys; P (A operand) from the S accumulators ----
#pragma unroll
    for (int ks = 0; ks < 4; ks++) {
      // A fragment rows g/g+8, keys 16ks + 2t, +1 (a0, a1) and +8, +9 (a2, a3): s tiles 2ks and 2ks+1
      const float* sa = s[2 * ks];
      const float* sb = s[2 * ks + 1];
      uint32_t ah[4], al[4];
      {
        const float v[8] = {sa[0], sa[1], sa[2], sa[3], sb[0], sb[1], sb[2], sb[3]};
        float hv[8], lv[8];
#pragma unroll
        for (int i = 0; i < 8; i++) {
          hv[i] = bf_round(v[i]);
          lv[i] = v[i] - hv[i];
        }
        ah[0] = bf2(hv[0], hv[1]);
        ah[1] = bf2(hv[2], hv[3]);
        ah[2] = bf2(hv[4], hv[5]);
        ah[3] = bf2(hv[6], hv[7]);
        al[0] = bf2(lv[0], lv[1]);
        al[1] = bf2(lv[2], lv[3]);
        al[2] = bf2(lv[4], lv[5]);
        al[3] = bf2(lv[6], lv[7]);
      }
#pragma unroll
      for (int np = 0; np < 8; np++) {  // 16 dims per ldmatrix.x4.trans: B (16 keys x 8 dims) x 2
        // matrices (keys 0-7|8-15) x (dims 0-7|8-15) of V stored [key][dim]
        const int m = lane >> 3, r = 16 * ks + (lane & 7) + 8 * (m & 1), c = 2 * np + (m >> 1);
        uint32_t b0, b1, b2, b3;
        ldsm4t(sv[cur] + swz(r, c), b0, b1, b2, b3);
        mma_bf16(o[2 * np], ah[0], ah[1], ah[2], ah[3], b0, b1);
        mma_bf16(o[2 * np], al[0], al[1], al[2], al[3], b0, b1);
        mma_bf16(o[2 * np + 1], ah[0], ah[1], ah[2], ah[3], b2, b3);
        mma_bf16(o[2 * np + 1], al[0], al[1], al[2], al[3], b2, b3);
      }
    }
    __syncthreads();  // tile `cur` may be refilled next iteration
  }
  cp_wait<0>();
  // ---- normalise and store (rows g, g+8; dims 8n + 2t, +1) ----
  const float i0 = l0 > 0.f ? 1.0f / l0 : 0.f, i1 = l1 > 0.f ? 1.0f / l1 : 0.f;
  float* ob = O + ((int64_t)b * Hq + h) * S * PA_D;
#pragma unroll
  for (int n = 0; n < 16; n++) {
    const int d = 8 * n + 2 * t;
    if (qr0 < S) *(float2*)(ob + (int64_t)qr0 * PA_D + d) = make_float2(o[n][0] * i0, o[n][1] * i0);
    if (qr1 < S) *(float2*)(ob + (int64_t)qr1 * PA_D + d) = make_float2(o[n][2] * i1, o[n][3] * i1);
  }
}

// ---------------------------------------------------------------------------
// tcgen05 flash attention.  One CTA = 128 queries (M) of one head, key tiles
// of 64 (N).  Warp 0: TMA (Q once, K and V^T tiles through a 3-stage ring);
// warp 1: tcgen05.mma issuer; warps 2-9: softmax, two threads per query row
// (TMEM lanes 32 (warp % 4) .. + 31), warps 2-5 on key columns 0-31 and
// output dims 0-63, warps 6-9 on the other halves; the two exchange their
// row maxima through shared memory.  Per key tile j:
//   S_j = Q K_j^T            (M 128, N 64, K 128: 8 MMAs) -> TMEM S[j % 2]
//   softmax: masked row max, p = exp(s - m), running sum, P_j written to
//            shared memory as bf16 hi + lo in the K-major 128-byte-swizzled
//            A-operand layout
//   O_j = P_hi V_j + P_lo V_j (M 128, N 128, K 64: 8 MMAs)  -> TMEM O[j % 2]
//   softmax warps: O += O_{j-1} rescaled (in registers), one tile behind.
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
// kind::f16 instruction descriptors: D f32, A and B bf16, both K-major
constexpr uint32_t FA_IDESC_S = (1u << 4) | (1u << 7) | (1u << 10) | ((64u >> 3) << 17) | ((128u >> 4) << 24);
constexpr uint32_t FA_IDESC_O = (1u << 4) | (1u << 7) | (1u << 10) | ((128u >> 3) << 17) | ((128u >> 4) << 24);

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
  // barriers: kv_full[NST] kv_empty[NST] s_full[2] s_free[2] p_full[2] o_full[2] o_free[2] q_full, TMEM slot
  const uint32_t kv_full = bars, kv_empty = bars + 8 * FA_NST, s_full = bars + 16 * FA_NST, s_free = s_full + 16,
                 p_full = s_full + 32, o_full = s_full + 48, o_free = s_full + 64, q_full = s_full + 80,
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
      mbar_init(o_free + 8 * i, 256);
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
                       sdesc_k128(sK + st * FA_KB + c * (FA_KB / 2)) + 2 * kk, FA_IDESC_S, (c | kk) != 0);
        }
        umma_commit(s_full + 8 * (j & 1));
      };
      if (nt > 0) issue_s(0);
      for (int j = 0; j < nt; j++) {
        if (j + 1 < nt) issue_s(j + 1);
        const int st = j % FA_NST, pb = j & 1;
        if (ok && !mbar_wait_bounded(p_full + 8 * pb, (uint32_t)((j / 2) & 1))) ok = false;
        if (ok && j >= 2 && !mbar_wait_bounded(o_free + 8 * pb, (uint32_t)((j / 2 - 1) & 1))) ok = false;
        tc_fence_after();
        if (ok) {
          const uint32_t ph = sP + pb * 2 * FA_PB, vt = sV + st * FA_VB, d = tmem + 128 + 128 * pb;
#pragma unroll
          for (int kk = 0; kk < 4; kk++)
            umma_f16(d, sdesc_k128(ph) + 2 * kk, sdesc_k128(vt) + 2 * kk, FA_IDESC_O, kk != 0);
#pragma unroll
          for (int kk = 0; kk < 4; kk++)
            umma_f16(d, sdesc_k128(ph + FA_PB) + 2 * kk, sdesc_k128(vt) + 2 * kk, FA_IDESC_O, 1);
        }
        umma_commit(o_full + 8 * pb);
        umma_commit(kv_empty + 8 * st);
      }
      if (!ok) atomicOr(err, SI_DEVERR_WAIT_TIMEOUT);
    }
  } else {  // softmax: two threads per query row r of the tile
    const int qq = warp & 3, half = (warp - 2) >> 2, r = 32 * qq + lane, qrow = q0 + r;
    const uint32_t lanes = (uint32_t)(32 * qq) << 16;
    float oacc[64];  // output dims 64 half .. + 63
#pragma unroll
    for (int i = 0; i < 64; i++) oacc[i] = 0.f;
    float m = -INFINITY, l = 0.f, alpha_prev = 1.f;  // m in base-2 units; l over this thread's keys
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
      // mask, running max (FlashAttention.cs:206-224, 238-325), in base-2
      // units: t = s * scale * log2(e), p = 2^(t - max t) = e^(s scale - max)
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
      asm volatile("bar.sync 1, 256;" ::: "memory");
      mx = fmaxf(mx, xch[pb * 256 + (half ^ 1) * 128 + r]);
      const float mn = fmaxf(m, mx);
      const float alpha = mn == -INFINITY ? 1.f : exp2f(m - mn);
      float ps = 0.f;
      if (mn != -INFINITY) {
#pragma unroll
        for (int i = 0; i < 32; i++) {
          const float p = exp2f(sv[i] - mn);  // 2^-inf = 0 for masked keys
          sv[i] = p;
          ps += p;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; i++) sv[i] = 0.f;
      }
      l = l * alpha + ps;
      m = mn;
      // P_j goes to the buffer P_{j-2} used; that product was complete when
      // O_{j-2} was added in the previous iteration
      {  // P_j as bf16 hi + lo: row r, chunks of 8 keys, chunk g at (g ^ (r % 8)) * 16 in the 128-byte row
        const uint32_t ph = sP + pb * 2 * FA_PB + r * 128;
#pragma unroll
        for (int gg = 0; gg < 4; gg++) {
          const int g = 4 * half + gg;
          uint32_t hi[4], lo[4];
#pragma unroll
          for (int e = 0; e < 4; e++) {
            const float a0 = sv[8 * gg + 2 * e], a1 = sv[8 * gg + 2 * e + 1];
            const __nv_bfloat162 h = __floats2bfloat162_rn(a0, a1);
            const float2 hf = __bfloat1622float2(h);
            const __nv_bfloat162 lw = __floats2bfloat162_rn(a0 - hf.x, a1 - hf.y);
            hi[e] = *(const uint32_t*)&h;
            lo[e] = *(const uint32_t*)&lw;
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
      if (j >= 1) {  // O += rescaled O_{j-1}
        if (ok && !mbar_wait_bounded(o_full + 8 * ((j - 1) & 1), (uint32_t)(((j - 1) / 2) & 1))) ok = false;
        tc_fence_after();
        const uint32_t ob = tmem + lanes + 128 + 128 * ((j - 1) & 1) + 64 * half;
#pragma unroll
        for (int c = 0; c < 2; c++) {
          uint32_t t32[32];
          tmem_ld32(ob + 32 * c, t32);
#pragma unroll
          for (int i = 0; i < 32; i++) oacc[32 * c + i] = fmaf(oacc[32 * c + i], alpha_prev, __uint_as_float(t32[i]));
        }
        tc_fence_before();
        mbar_arrive(o_free + 8 * ((j - 1) & 1));
      }
      alpha_prev = alpha;
    }
    if (nt > 0) {  // the last tile's O
      const int j = nt - 1;
      if (ok && !mbar_wait_bounded(o_full + 8 * (j & 1), (uint32_t)((j / 2) & 1))) ok = false;
      tc_fence_after();
      const uint32_t ob = tmem + lanes + 128 + 128 * (j & 1) + 64 * half;
#pragma unroll
      for (int c = 0; c < 2; c++) {
        uint32_t t32[32];
        tmem_ld32(ob + 32 * c, t32);
#pragma unroll
        for (int i = 0; i < 32; i++) oacc[32 * c + i] = fmaf(oacc[32 * c + i], alpha_prev, __uint_as_float(t32[i]));
      }
    }
    xch[512 + half * 128 + r] = l;  // the row sum adds both halves' keys
    asm volatile("bar.sync 1, 256;" ::: "memory");
    const float lr = l + xch[512 + (half ^ 1) * 128 + r];
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

// 3D bf16 tensor [n2][n1][n0] (n0 contiguous), box [b2 = 1][b1][64], 128-byte swizzle.
int make_tmap3(CUtensorMap* tm, const void* ptr, int64_t n0, int64_t n1, int64_t n2, int b1) {
  auto fn = encode_fn();
  if (!fn) SI_FAIL(SI_ERR_CUDA, "si_attn_prefill: cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[3] = {(cuuint64_t)n0, (cuuint64_t)n1, (cuuint64_t)n2};
  const cuuint64_t strides[2] = {(cuuint64_t)n0 * 2, (cuuint64_t)n0 * n1 * 2};
  const cuuint32_t box[3] = {64, (cuuint32_t)b1, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) SI_FAIL(SI_ERR_CUDA, "si_attn_prefill: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return SI_OK;
}

}  // namespace
}  // namespace si

using namespace si;

extern "C" SI_EXPORT int si_attn_prefill(si_ctx* c, const uint16_t* q, const uint16_t* k, const uint16_t* v, float* o,
                                         int batch, int heads, int kv_heads, int seq, int kv, int head_dim,
                                         float scale, int causal, int start_pos) {
  clear_error();
  if (!c || !q || !k || !v || !o) SI_FAIL(SI_ERR_INVALID, "si_attn_prefill: NULL argument");
  if (head_dim != PA_D) SI_FAIL(SI_ERR_UNSUPPORTED, "si_attn_prefill: head_dim %d (this build supports 128)", head_dim);
  if (batch < 1 || heads < 1 || kv_heads < 1 || heads % kv_heads || seq < 1 || kv < 0)
    SI_FAIL(SI_ERR_INVALID, "si_attn_prefill: bad shape");
  if (batch > 65535 || heads > 65535) SI_FAIL(SI_ERR_UNSUPPORTED, "si_attn_prefill: batch/heads above 65535");
  if (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)o) & 15)
    SI_FAIL(SI_ERR_INVALID, "si_attn_prefill: buffers must be 16-byte aligned");
  SI_TRY(bind_device(c));
  if (kv > 0) {  // tensor cores (tcgen05): V transposed into scratch, Q/K/V^T through TMA
    const int kvp = (kv + 7) & ~7;  // 16-byte rows of V^T
    SI_TRY(ensure(c->stage[3], (size_t)batch * kv_heads * PA_D * kvp * 2));
    uint16_t* vt = (uint16_t*)c->stage[3].ptr;
    k_vt<<<dim3((unsigned)((kvp + 31) / 32), PA_D / 32, (unsigned)(batch * kv_heads)), dim3(32, 8), 0, c->stream>>>(
        v, vt, kv, kvp);
    SI_CUDA(cudaGetLastError());
    CUtensorMap tq, tk, tv;
    SI_TRY(make_tmap3(&tq, q, PA_D, seq, (int64_t)batch * heads, FA_BQ));
    SI_TRY(make_tmap3(&tk, k, PA_D, kv, (int64_t)batch * kv_heads, FA_BK));
    SI_TRY(make_tmap3(&tv, vt, kvp, PA_D, (int64_t)batch * kv_heads, PA_D));
    static uint64_t fa_attr = 0;
    if (c->device < 64 && !(fa_attr & (1ull << c->device))) {
      SI_CUDA(cudaFuncSetAttribute(k_attn_fa_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, FA_SMEM));
      fa_attr |= 1ull << c->device;
    }
    dim3 grid((unsigned)((seq + FA_BQ - 1) / FA_BQ), (unsigned)heads, (unsigned)batch);
    k_attn_fa_tc<<<grid, FA_THREADS, FA_SMEM, c->stream>>>(tq, tk, tv, o, heads, kv_heads, seq, kv, scale, causal,
                                                    start_pos, c->dev_err);
    SI_CUDA(cudaGetLastError());
    return SI_OK;
  }
  const int smem = 5 * PA_TILE;
  static uint64_t attr_set = 0;
  if (c->device < 64 && !(attr_set & (1ull << c->device))) {
    SI_CUDA(cudaFuncSetAttribute(k_attn_prefill, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr_set |= 1ull << c->device;
  }
  dim3 grid((unsigned)((seq + PA_BQ - 1) / PA_BQ), (unsigned)heads, (unsigned)batch);
  k_attn_prefill<<<grid, 128, smem, c->stream>>>((const __nv_bfloat16*)q, (const __nv_bfloat16*)k,
                                                  (const __nv_bfloat16*)v, o, heads, kv_heads, seq, kv, scale, causal,
                                                  start_pos);
  SI_CUDA(cudaGetLastError());
  return SI_OK;
}
