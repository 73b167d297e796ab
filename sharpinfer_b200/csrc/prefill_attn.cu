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
#include <cuda_bf16.h>

#include "common.cuh"

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
