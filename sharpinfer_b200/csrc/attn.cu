// Decode attention over the f16 KV cache: RoPE, KV append and split-KV
// flash-decoding with an online-softmax merge.
//
// Semantics follow the attention block of Transformer.Forward
// (src/SharpInfer.Core/Layers/Transformer.cs:94-129): RotaryEmbedding.Apply
// on q and k (RotaryEmbedding.cs:24-61, adjacent pairs, angles taken from a
// host-computed cos/sin table with the reference's float formula),
// KVCache.Store (KVCache.cs:46-57) of the roped k and v -- rounded to f16, the
// device cache's type -- then for every q head h with kv head h / (nh/nkv):
// softmax over t <= pos of Dot(q_h, K_t) * (1/sqrt(hd)) and the weighted sum
// of V_t.
//
// Cache layout: [layer][seq][kv head][position][128] f16, so the positions of
// one (seq, kv head) are contiguous and a 64-position chunk is one 16 KB bulk
// copy.  Grid (split, kv head, seq): CTA s handles positions
// [s*chunk, min(len, (s+1)*chunk)), len = pos + 1.  Its 8 warps first score
// all its positions for the G = nh/nkv q heads of the kv head, then
// accumulate p * V; K and V chunks stream through a shared-memory ring filled
// by thread 0 (cp.async.bulk + mbarriers, bounded waits).  Each CTA writes
// (max, sum, o[128]) per head; the last CTA of a (seq, kv head) merges them.
#include "common.cuh"
#include "model.cuh"

namespace si {
namespace {

constexpr int HD = 128;
constexpr int AT_WARPS = 8;
constexpr int AT_SUB = 64;                 // positions per ring stage
constexpr int AT_NS = 4;                   // ring stages
constexpr int AT_STAGE = AT_SUB * HD * 2;  // 16 KB
constexpr int AT_QSTRIDE = 36;             // floats per 32-dim quarter of q (padded)

__device__ __forceinline__ float f16lo(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w & 0xFFFF))); }
__device__ __forceinline__ float f16hi(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w >> 16))); }

struct AttnSmem {
  // ring of K/V chunks, then q, scores, partial outputs, barriers
  static constexpr int RING = AT_NS * AT_STAGE;
};

template <int G>
__global__ void __launch_bounds__(AT_WARPS * 32) k_attn_decode(AttnArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int s_idx = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int S = gridDim.x, nkv = gridDim.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint8_t* ring = smem;
  const int cpad = (a.chunk_max + 3) & ~3;                 // keeps the next region 16-B aligned
  float* qs = (float*)(smem + AttnSmem::RING);           // [G][4][AT_QSTRIDE]
  float* sc = qs + G * 4 * AT_QSTRIDE;                    // [G][cpad]
  float* ored = sc + G * cpad;                            // [AT_WARPS][G][HD]
  float* stat = ored + AT_WARPS * G * HD;                 // [G][2] max, sum + flag
  uint64_t* bars = (uint64_t*)(stat + 2 * G + 2);         // aligned below
  bars = (uint64_t*)(((uintptr_t)bars + 7) & ~(uintptr_t)7);
  const uint32_t bar0 = smem_u32(bars);

  pdl_wait();
  const int pos = a.params->pos;
  const int len = pos + 1;
  const int chunk = (len + S - 1) / S;
  const int t0 = s_idx * chunk, t1 = min(len, t0 + chunk);
  const int n = max(0, t1 - t0);
  const int nsub = (n + AT_SUB - 1) / AT_SUB;
  const int64_t cache_off = (((int64_t)a.layer * a.max_batch + b) * nkv + kvh) * a.max_seq * HD;
  __half* kc = a.kcache + cache_off;
  __half* vc = a.vcache + cache_off;
  const float* qkv = a.qkv + (int64_t)b * a.qkv_ld;
  const float2* rope = (const float2*)(a.rope + (int64_t)pos * HD);  // [HD/2] (cos, sin)

  // q heads of this kv head, roped (RotaryEmbedding.ApplyToHead), into smem
  for (int i = tid; i < G * HD / 2; i += blockDim.x) {
    const int h = i / (HD / 2), p = i % (HD / 2);
    const float* qh = qkv + (int64_t)(kvh * G + h) * HD;
    const float x0 = qh[2 * p], x1 = qh[2 * p + 1];
    const float2 cs = rope[p];
    const float r0 = __fsub_rn(__fmul_rn(x0, cs.x), __fmul_rn(x1, cs.y));
    const float r1 = __fadd_rn(__fmul_rn(x0, cs.y), __fmul_rn(x1, cs.x));
    const int d0 = 2 * p;
    qs[(h * 4 + (d0 >> 5)) * AT_QSTRIDE + (d0 & 31)] = r0;
    qs[(h * 4 + ((d0 + 1) >> 5)) * AT_QSTRIDE + ((d0 + 1) & 31)] = r1;
  }
  // the split holding `pos` appends the roped k and v (KVCache.Store)
  if (t1 == len && n > 0 && tid < HD / 2) {
    const int p = tid;
    const float* kh = qkv + (int64_t)(a.nh + kvh) * HD;
    const float* vh = qkv + (int64_t)(a.nh + nkv + kvh) * HD;
    const float2 cs = rope[p];
    const float x0 = kh[2 * p], x1 = kh[2 * p + 1];
    const float r0 = __fsub_rn(__fmul_rn(x0, cs.x), __fmul_rn(x1, cs.y));
    const float r1 = __fadd_rn(__fmul_rn(x0, cs.y), __fmul_rn(x1, cs.x));
    *(__half2*)(kc + (int64_t)pos * HD + 2 * p) = __halves2half2(__float2half_rn(r0), __float2half_rn(r1));
    *(__half2*)(vc + (int64_t)pos * HD + 2 * p) =
        __halves2half2(__float2half_rn(vh[2 * p]), __float2half_rn(vh[2 * p + 1]));
    // make these generic-proxy writes visible to the bulk (async-proxy) reads below
    asm volatile("fence.proxy.async.global;" ::: "memory");
  }
  if (tid == 0) {
    for (int i = 0; i < AT_NS; i++) mbar_init(bar0 + 8 * i, 1);
    mbar_fence_init();
  }
  __syncthreads();

  // ring items: K sub-chunks 0..nsub-1, then V sub-chunks 0..nsub-1
  const int items = 2 * nsub;
  auto issue = [&](int it) {
    const int st = it % AT_NS;
    const int sub = it < nsub ? it : it - nsub;
    const __half* base = it < nsub ? kc : vc;
    const int p0 = t0 + sub * AT_SUB;
    const int np = min(AT_SUB, t1 - p0);
    const uint32_t bytes = (uint32_t)np * HD * 2;
    mbar_arrive_expect_tx(bar0 + 8 * st, bytes);
    bulk_g2s(smem_u32(ring + st * AT_STAGE), base + (int64_t)p0 * HD, bytes, bar0 + 8 * st);
  };
  if (tid == 0)
    for (int it = 0; it < min(items, AT_NS); it++) issue(it);

  bool ok = true;
  const float scale = a.scale;
  // ---- pass 1: scores ----
  // warp handles 8 positions per step: lane (pp = lane/4, quarter qq = lane%4)
  const int pp = lane >> 2, qq = lane & 3;
  for (int it = 0; it < nsub; it++) {
    const int st = it % AT_NS;
    if (!mbar_wait_bounded(bar0 + 8 * st, (uint32_t)((it / AT_NS) & 1))) ok = false;
    const int p0 = t0 + it * AT_SUB;
    const int np = min(AT_SUB, t1 - p0);
    const uint8_t* kst = ring + st * AT_STAGE;
    for (int tl = warp * 8 + pp; tl < AT_SUB; tl += AT_WARPS * 8) {
      float acc[G];
#pragma unroll
      for (int h = 0; h < G; h++) acc[h] = 0.f;
      if (tl < np && ok) {
        const uint4* kr = (const uint4*)(kst + tl * HD * 2 + qq * 64);
        float kf[32];
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const uint4 v = kr[i];
          kf[8 * i + 0] = f16lo(v.x); kf[8 * i + 1] = f16hi(v.x);
          kf[8 * i + 2] = f16lo(v.y); kf[8 * i + 3] = f16hi(v.y);
          kf[8 * i + 4] = f16lo(v.z); kf[8 * i + 5] = f16hi(v.z);
          kf[8 * i + 6] = f16lo(v.w); kf[8 * i + 7] = f16hi(v.w);
        }
#pragma unroll
        for (int h = 0; h < G; h++) {
          const float4* q4 = (const float4*)(qs + (h * 4 + qq) * AT_QSTRIDE);
          float d = 0.f;
#pragma unroll
          for (int i = 0; i < 8; i++) {
            const float4 qv = q4[i];
            d = fmaf(qv.x, kf[4 * i + 0], d);
            d = fmaf(qv.y, kf[4 * i + 1], d);
            d = fmaf(qv.z, kf[4 * i + 2], d);
            d = fmaf(qv.w, kf[4 * i + 3], d);
          }
          acc[h] = d;
        }
      }
#pragma unroll
      for (int h = 0; h < G; h++) {
        float d = acc[h];
        d += __shfl_xor_sync(0xFFFFFFFFu, d, 1);
        d += __shfl_xor_sync(0xFFFFFFFFu, d, 2);
        if (qq == 0 && tl < np) sc[h * cpad + it * AT_SUB + tl] = d * scale;
      }
    }
    __syncthreads();  // stage consumed by every warp
    if (tid == 0 && it + AT_NS < items) issue(it + AT_NS);
  }
  // ---- softmax statistics per head (TensorOps.Softmax: max, exp, sum) ----
  for (int h = warp; h < G; h += AT_WARPS) {
    float m = -INFINITY;
    for (int i = lane; i < n; i += 32) m = fmaxf(m, sc[h * cpad + i]);
    m = warp_max(m);
    float l = 0.f;
    for (int i = lane; i < n; i += 32) {
      const float p = expf(sc[h * cpad + i] - m);
      sc[h * cpad + i] = p;
      l += p;
    }
    l = warp_sum(l);
    if (lane == 0) {
      stat[2 * h] = n > 0 ? m : -INFINITY;
      stat[2 * h + 1] = l;
    }
  }
  __syncthreads();
  // ---- pass 2: o[h][d] = sum_t p[h][t] * V_t[d]; lane holds dims 4*lane..+3 ----
  float o[G][4];
#pragma unroll
  for (int h = 0; h < G; h++) o[h][0] = o[h][1] = o[h][2] = o[h][3] = 0.f;
  for (int it = nsub; it < items; it++) {
    const int st = it % AT_NS;
    if (!mbar_wait_bounded(bar0 + 8 * st, (uint32_t)((it / AT_NS) & 1))) ok = false;
    const int sub = it - nsub;
    const int np = min(AT_SUB, t1 - (t0 + sub * AT_SUB));
    const uint8_t* vst = ring + st * AT_STAGE;
    if (ok) {
      for (int tl = warp; tl < np; tl += AT_WARPS) {
        const uint2 v = *(const uint2*)(vst + tl * HD * 2 + lane * 8);
        const float v0 = f16lo(v.x), v1 = f16hi(v.x), v2 = f16lo(v.y), v3 = f16hi(v.y);
#pragma unroll
        for (int h = 0; h < G; h++) {
          const float p = sc[h * cpad + sub * AT_SUB + tl];
          o[h][0] = fmaf(p, v0, o[h][0]);
          o[h][1] = fmaf(p, v1, o[h][1]);
          o[h][2] = fmaf(p, v2, o[h][2]);
          o[h][3] = fmaf(p, v3, o[h][3]);
        }
      }
    }
    __syncthreads();
    if (tid == 0 && it + AT_NS < items) issue(it + AT_NS);
  }
  // reduce the 8 warps' partial outputs
#pragma unroll
  for (int h = 0; h < G; h++)
    *(float4*)(ored + (warp * G + h) * HD + lane * 4) = make_float4(o[h][0], o[h][1], o[h][2], o[h][3]);
  __syncthreads();
  const int64_t pbase = (((int64_t)b * a.nh + kvh * G) * S + s_idx);  // head h: + h*S
  for (int i = tid; i < G * HD; i += blockDim.x) {
    const int h = i / HD, d = i % HD;
    float v = 0.f;
    for (int w = 0; w < AT_WARPS; w++) v += ored[(w * G + h) * HD + d];
    a.part_o[(pbase + (int64_t)h * S) * HD + d] = v;
  }
  if (tid < G) {
    a.part_ml[(pbase + (int64_t)tid * S) * 2 + 0] = stat[2 * tid];
    a.part_ml[(pbase + (int64_t)tid * S) * 2 + 1] = stat[2 * tid + 1];
  }
  if (!ok && tid == 0) atomicOr(a.err, SI_DEVERR_WAIT_TIMEOUT);
  // ---- last CTA of (seq, kv head) merges the S partials ----
  __threadfence();
  __syncthreads();
  int* cnt = a.counters + (int64_t)b * nkv + kvh;
  if (tid == 0) stat[2 * G] = (float)atomicAdd(cnt, 1);
  __syncthreads();
  if (stat[2 * G] == (float)(S - 1)) {
    // Partials of the other CTAs are read through L2 (ld.global.cg) after the
    // fence: their statistics first, then all S partial outputs of a
    // (head, dim) pair with the loads of one thread independent of each other.
    __threadfence();
    float* pm = ored;           // [G][S] partial max, then merge weight
    float* pl = ored + G * S;   // [G][S] partial sum
    float* inv = pl + G * S;    // [G] 1 / merged denominator
    for (int i = tid; i < G * S; i += blockDim.x) {
      const int h = i / S, s = i - h * S;
      const int64_t e = ((int64_t)b * a.nh + kvh * G + h) * S + s;
      pm[i] = __ldcg(a.part_ml + e * 2);
      pl[i] = __ldcg(a.part_ml + e * 2 + 1);
    }
    __syncthreads();
    for (int h = warp; h < G; h += AT_WARPS) {
      float M = -INFINITY;
      for (int s = lane; s < S; s += 32) M = fmaxf(M, pm[h * S + s]);
      M = warp_max(M);
      float den = 0.f;
      for (int s = lane; s < S; s += 32) {
        const float m = pm[h * S + s];
        const float w = m == -INFINITY ? 0.f : expf(m - M);
        pm[h * S + s] = w;
        den = fmaf(w, pl[h * S + s], den);
      }
      den = warp_sum(den);
      if (lane == 0) inv[h] = 1.0f / den;
    }
    __syncthreads();
    for (int i = tid; i < G * HD; i += blockDim.x) {
      const int h = i / HD, d = i % HD;
      const float* po = a.part_o + ((int64_t)b * a.nh + kvh * G + h) * S * HD + d;
      const float* wh = pm + h * S;
      float num0 = 0.f, num1 = 0.f, num2 = 0.f, num3 = 0.f;
      int s = 0;
      for (; s + 4 <= S; s += 4) {
        num0 = fmaf(wh[s], __ldcg(po + (int64_t)s * HD), num0);
        num1 = fmaf(wh[s + 1], __ldcg(po + (int64_t)(s + 1) * HD), num1);
        num2 = fmaf(wh[s + 2], __ldcg(po + (int64_t)(s + 2) * HD), num2);
        num3 = fmaf(wh[s + 3], __ldcg(po + (int64_t)(s + 3) * HD), num3);
      }
      for (; s < S; s++) num0 = fmaf(wh[s], __ldcg(po + (int64_t)s * HD), num0);
      a.out[(int64_t)b * a.out_ld + (int64_t)(kvh * G + h) * HD + d] = ((num0 + num1) + (num2 + num3)) * inv[h];
    }
    if (tid == 0) *cnt = 0;
  }
  pdl_launch();
}

}  // namespace

size_t attn_smem_bytes(int G, int chunk_max) {
  const int cpad = (chunk_max + 3) & ~3;
  return (size_t)AT_NS * AT_STAGE + (size_t)G * 4 * AT_QSTRIDE * 4 + (size_t)G * cpad * 4 +
         (size_t)AT_WARPS * G * HD * 4 + (2 * G + 2) * 4 + 8 + AT_NS * 8;
}

int launch_attn(cudaStream_t s, const AttnArgs& a, int G, int splits, int batch, int nkv, bool pdl) {
  const size_t smem = attn_smem_bytes(G, a.chunk_max);
  if (smem > 227 * 1024) SI_FAIL(SI_ERR_UNSUPPORTED, "attention: %zu bytes of shared memory needed", smem);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(splits, nkv, batch);
  cfg.blockDim = dim3(AT_WARPS * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  switch (G) {
#define SI_ATTN_CASE(GG)                                                                      \
  case GG:                                                                                    \
    SI_CUDA(cudaFuncSetAttribute(k_attn_decode<GG>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                 (int)smem));                                                 \
    SI_CUDA(cudaLaunchKernelEx(&cfg, k_attn_decode<GG>, a));                                  \
    return SI_OK;
    SI_ATTN_CASE(1)
    SI_ATTN_CASE(2)
    SI_ATTN_CASE(4)
    SI_ATTN_CASE(8)
#undef SI_ATTN_CASE
    default:
      SI_FAIL(SI_ERR_UNSUPPORTED, "attention: %d q heads per kv head (supported 1, 2, 4, 8)", G);
  }
}

}  // namespace si
