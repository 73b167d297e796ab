// Decode attention over the f16 KV cache: RoPE, KV append and split-KV
// flash-decoding with an online-softmax merge, on the tensor cores.
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
// Cache layout: [layer][seq][kv head][position][128] f16 with the 16-byte
// chunks of each row XOR-swizzled by position (kv_swz), so the positions of
// one (seq, kv head) are contiguous and a 64-position chunk is one 16 KB bulk
// copy.  Grid (split, kv head, seq): CTA s handles positions
// [s*chunk, min(len, (s+1)*chunk)), len = pos + 1, with 4 warps, each taking
// one 16-position block of every 64-position ring stage:
//  * scores: mma.m16n8k16 with A = 16 cached K rows x 16 dims (ldmatrix) and
//    B = the G q heads split into f16 hi + lo columns (q scaled by a power of
//    two per head), f32 accumulation;
//  * softmax over the CTA's positions (max, expf, sum), probabilities stored
//    as f16 hi + lo;
//  * output: mma with A = V^T (ldmatrix.trans), B = the probabilities.
// Each CTA writes (max, sum, o[128]) per head; the kernel that prepares the
// O-projection input merges the splits (k_prep, SI_PREP_ATTN_MERGE).  CTAs
// whose positions are all in the cache already start their K/V copies before
// waiting for the kernel that produces q.
#include "common.cuh"
#include "model.cuh"
#include "prepfmt.cuh"

namespace si {
namespace {

constexpr int HD = 128;
constexpr int AT_WARPS = 4;
constexpr int AT_SUB = 64;                 // positions per ring stage (4 blocks of 16)
constexpr int AT_NS = 4;                   // ring stages (2 at batch >= 4: a third CTA fits per SM)
constexpr int AT_STAGE = AT_SUB * HD * 2;  // 16 KB

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& a0, uint32_t& a1, uint32_t& a2, uint32_t& a3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(a0), "=r"(a1), "=r"(a2), "=r"(a3)
               : "r"(addr)
               : "memory");
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& a0, uint32_t& a1, uint32_t& a2, uint32_t& a3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(a0), "=r"(a1), "=r"(a2), "=r"(a3)
               : "r"(addr)
               : "memory");
}
// f16 hi (part 0) or lo (part 1) of v, two values packed
__device__ __forceinline__ uint32_t split2(float v0, float v1, int part) {
  const __half h0 = __float2half_rn(v0), h1 = __float2half_rn(v1);
  if (part == 0) return (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
  const __half l0 = __float2half_rn(v0 - __half2float(h0)), l1 = __float2half_rn(v1 - __half2float(h1));
  return (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
}

struct AttnSmem {
  int G, cp, ns;  // heads per kv head, positions per split rounded up to 64, ring stages
  __host__ __device__ size_t qs() const { return (size_t)ns * AT_STAGE; }              // f32 [G][128]
  __host__ __device__ size_t qsc() const { return qs() + (size_t)G * HD * 4; }          // f32 [16]
  __host__ __device__ size_t sc() const { return qsc() + 64; }                          // f32 [G][cp]
  __host__ __device__ size_t pp() const { return sc() + (size_t)G * cp * 4; }           // f16 [2][G][cp]
  __host__ __device__ size_t ored() const { return pp() + (size_t)2 * G * cp * 2; }     // f32 [W][G][128]
  __host__ __device__ size_t stat() const { return ored() + (size_t)AT_WARPS * G * HD * 4; }  // f32 [G][2] + 2
  __host__ __device__ size_t bars() const { return (stat() + (2 * G + 2) * 4 + 7) & ~(size_t)7; }
  __host__ __device__ size_t total() const { return bars() + (size_t)ns * 8; }
};

// The last CTA of (sequence b, kv head kvh) to finish merges the S splits of
// its G heads -- the softmax of Transformer.cs:99-129 over all positions:
// M = max_s m_s, w_s = exp(m_s - M), o = sum_s w_s o_s / sum_s w_s l_s --
// and packs the G * 128 merged values (G / 2 whole 256-column units) as the
// O projection's prepared input.  Every CTA's partials are made visible
// (fence) before it counts itself in; the order of the sums is fixed, so the
// result does not depend on which CTA merges.  smem: the K/V ring, idle by now.
template <int G>
__device__ __forceinline__ void attn_merge_last(const AttnArgs& a, uint8_t* smem, int b, int kvh, int S) {
  __shared__ int is_last;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  __threadfence();
  __syncthreads();
  int* cnt = a.merge_cnt + b * gridDim.y + kvh;
  if (tid == 0) is_last = atomicAdd(cnt, 1) == S - 1;
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  static_assert(8 * SI_ATTN_MAX_SPLITS * 4 <= 16384 && 16640 + 8 * HD * 4 <= 2 * AT_STAGE, "merge scratch");
  float* wts = (float*)smem;                        // [G][S] merge weights
  float* inv = (float*)(smem + 16384);              // [G] 1 / sum_s w_s l_s
  float* sv = (float*)(smem + 16640);               // [G][128] merged values (16-byte aligned)
  const int64_t hb = (int64_t)b * a.nh + kvh * G;   // first head of the group, this sequence
  for (int h = warp; h < G; h += AT_WARPS) {
    const float2* ml = (const float2*)a.part_ml + (hb + h) * S;
    float M = -INFINITY;
    for (int s = lane; s < S; s += 32) M = fmaxf(M, __ldcg(ml + s).x);
    M = warp_max(M);
    float den = 0.f;
    for (int s = lane; s < S; s += 32) {
      const float2 v = __ldcg(ml + s);
      const float w = v.x == -INFINITY ? 0.f : expf(v.x - M);
      wts[h * SI_ATTN_MAX_SPLITS + s] = w;
      den = fmaf(w, v.y, den);
    }
    den = warp_sum(den);
    if (lane == 0) inv[h] = 1.0f / den;
  }
  __syncthreads();
  for (int i = tid; i < G * 32; i += blockDim.x) {  // (head, 4 dims) per thread
    const int h = i >> 5, d4 = i & 31;
    const float4* po = (const float4*)(a.part_o + (hb + h) * S * HD) + d4;
    const float* wh = wts + h * SI_ATTN_MAX_SPLITS;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s0 = 0; s0 < S; s0 += 16) {  // 16 partial outputs in flight
      float4 o[16];
#pragma unroll
      for (int j = 0; j < 16; j++)
        if (s0 + j < S) o[j] = __ldcg(po + (int64_t)(s0 + j) * (HD / 4));
#pragma unroll
      for (int j = 0; j < 16; j++)
        if (s0 + j < S) {
          const float w = wh[s0 + j];
          acc.x = fmaf(w, o[j].x, acc.x);
          acc.y = fmaf(w, o[j].y, acc.y);
          acc.z = fmaf(w, o[j].z, acc.z);
          acc.w = fmaf(w, o[j].w, acc.w);
        }
    }
    const float r = inv[h];
    const float4 v = make_float4(acc.x * r, acc.y * r, acc.z * r, acc.w * r);
    *(float4*)(sv + h * HD + 4 * d4) = v;
    if (a.out) *(float4*)(a.out + (hb + h) * HD + 4 * d4) = v;
  }
  __syncthreads();
  // prepared units: the group's heads cover units kvh * G / 2 .. + G / 2 - 1
  const int B = gridDim.z, nunit = a.nh * HD / 256, mg = b >> 2, cb = b & 3;
  const int LW = 8 * min(4, B - 4 * mg);
  for (int u = warp; u < G / 2; u += AT_WARPS)
    pack_unit_warp(sv + 256 * u, a.xprep + xprep_off(mg, nunit, kvh * (G / 2) + u, LW), LW, cb, lane);
  if (tid == 0) *cnt = 0;
}

template <int G, int NS>
__global__ void __launch_bounds__(AT_WARPS * 32) k_attn_decode(AttnArgs a) {
  constexpr int NT = (2 * G + 7) / 8;  // n-tiles of 8 (head, hi/lo) columns
  extern __shared__ __align__(128) uint8_t smem[];
  const int s_idx = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int S = gridDim.x, nkv = gridDim.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const AttnSmem L{G, (a.chunk_max + 63) & ~63, NS};
  const int cp = L.cp;
  uint8_t* ring = smem;
  float* qs = (float*)(smem + L.qs());
  float* qsc = (float*)(smem + L.qsc());  // [0, G): score factor, [8, 8 + G): q multiplier
  float* sc = (float*)(smem + L.sc());
  uint16_t* pp = (uint16_t*)(smem + L.pp());
  float* ored = (float*)(smem + L.ored());
  float* stat = (float*)(smem + L.stat());
  const uint32_t bar0 = smem_u32(smem + L.bars());

  pdl_launch();  // dependents may start their independent prologue now
  // The position comes from the step parameters, which no kernel of the step
  // writes, and positions < pos are already in the cache: both may be read
  // before the producer of q has finished.
  const int pos = a.params->pos;
  const int len = pos + 1;
  // The last split holds only the newest (up to) 16 positions, the one being
  // appended among them: the CTA that stores position pos copies its K/V only
  // after that store, so it gets the least to copy.  The other splits share
  // the rest evenly.
  const int tail = S > 1 ? min(16, len) : len;
  const int chunk = S > 1 ? (len - tail + S - 2) / (S - 1) : len;
  const int t0 = s_idx == S - 1 ? len - tail : s_idx * chunk;
  const int t1 = s_idx == S - 1 ? len : min(len - tail, t0 + chunk);
  const int n = max(0, t1 - t0);
  const int nsub = (n + AT_SUB - 1) / AT_SUB;
  const bool appends = t1 == len && n > 0;  // this split stores position pos
  const int64_t cache_off = (((int64_t)a.layer * a.max_batch + b) * nkv + kvh) * a.max_seq * HD;
  __half* kc = a.kcache + cache_off;
  __half* vc = a.vcache + cache_off;
  if (tid == 0) {
    for (int i = 0; i < NS; i++) mbar_init(bar0 + 8 * i, 1);
    mbar_fence_init();
  }
  __syncthreads();
  // ring items: K sub-chunks 0..nsub-1, then V sub-chunks 0..nsub-1
  const int items = 2 * nsub;
  const uint64_t pol = l2_evict_first_policy();  // the cache is read once per step
  auto issue = [&](int it) {
    const int st = it % NS;
    const int sub = it < nsub ? it : it - nsub;
    const __half* base = it < nsub ? kc : vc;
    const int p0 = t0 + sub * AT_SUB;
    const int np = min(AT_SUB, t1 - p0);
    const uint32_t bytes = (uint32_t)np * HD * 2;
    mbar_arrive_expect_tx(bar0 + 8 * st, bytes);
    bulk_g2s_ef(smem_u32(ring + st * AT_STAGE), base + (int64_t)p0 * HD, bytes, bar0 + 8 * st, pol);
  };
  if (tid == 0 && !appends)
    for (int it = 0; it < min(items, NS); it++) issue(it);
  l2_prefetch_share(a.pf);
  pdl_wait();
  const float* qkv = a.qkv + (int64_t)b * a.qkv_ld;
  const float2* rope = (const float2*)(a.rope + (int64_t)pos * HD);  // [HD/2] (cos, sin)

  // q heads of this kv head, roped (RotaryEmbedding.ApplyToHead), into smem
  for (int i = tid; i < G * HD / 2; i += blockDim.x) {
    const int h = i / (HD / 2), p = i % (HD / 2);
    const float* qh = qkv + (int64_t)(kvh * G + h) * HD;
    const float x0 = qh[2 * p], x1 = qh[2 * p + 1];
    const float2 cs = rope[p];
    qs[h * HD + 2 * p] = __fsub_rn(__fmul_rn(x0, cs.x), __fmul_rn(x1, cs.y));
    qs[h * HD + 2 * p + 1] = __fadd_rn(__fmul_rn(x0, cs.y), __fmul_rn(x1, cs.x));
  }
  // the split holding `pos` appends the roped k and v (KVCache.Store), then
  // starts its copies
  if (appends && tid < HD / 2) {
    const int p = tid;
    const float* kh = qkv + (int64_t)(a.nh + kvh) * HD;
    const float* vh = qkv + (int64_t)(a.nh + nkv + kvh) * HD;
    const float2 cs = rope[p];
    const float x0 = kh[2 * p], x1 = kh[2 * p + 1];
    const float r0 = __fsub_rn(__fmul_rn(x0, cs.x), __fmul_rn(x1, cs.y));
    const float r1 = __fadd_rn(__fmul_rn(x0, cs.y), __fmul_rn(x1, cs.x));
    const int o = kv_swz(2 * p, pos);  // dims 2p, 2p+1 stay adjacent
    *(__half2*)(kc + (int64_t)pos * HD + o) = __halves2half2(__float2half_rn(r0), __float2half_rn(r1));
    *(__half2*)(vc + (int64_t)pos * HD + o) = __halves2half2(__float2half_rn(vh[2 * p]), __float2half_rn(vh[2 * p + 1]));
    // make these generic-proxy writes visible to the bulk (async-proxy) reads below
    asm volatile("fence.proxy.async.global;" ::: "memory");
  }
  __syncthreads();
  if (tid == 0 && appends)
    for (int it = 0; it < min(items, NS); it++) issue(it);

  // per-head power-of-two scale of q: max |q 2^e| in [2^13, 2^14)
  for (int h = warp; h < G; h += AT_WARPS) {
    float m = 0.f;
    for (int d = lane; d < HD; d += 32) m = fmaxf(m, fabsf(qs[h * HD + d]));
    m = warp_max(m);
    const int e = unit_exponent(m);
    if (lane == 0) {
      qsc[h] = a.scale * exp2i(-e);
      qsc[8 + h] = exp2i(e);
    }
  }
  __syncthreads();
  // q B fragments: column n = g is (head 4 nt + g/2, part g%2)
  uint32_t qb[NT][8][2];
#pragma unroll
  for (int nt = 0; nt < NT; nt++) {
    const int h = 4 * nt + (g >> 1), part = g & 1;
#pragma unroll
    for (int ks = 0; ks < 8; ks++) {
      if (h < G) {
        const float mul = qsc[8 + h];
        const float* q = qs + h * HD + 16 * ks + 2 * t;
        qb[nt][ks][0] = split2(q[0] * mul, q[1] * mul, part);
        qb[nt][ks][1] = split2(q[8] * mul, q[9] * mul, part);
      } else {
        qb[nt][ks][0] = qb[nt][ks][1] = 0u;
      }
    }
  }

  bool ok = true;
  // After a wait gives up (agreed by the whole CTA at the stage's barrier)
  // nothing more is issued; thread 0 waits once, bounded, on each item still
  // in flight -- items it .. it + NS - 1 -- and the CTA skips the rest.
  auto drain = [&](int it) {
    if (tid == 0)
      for (int j = it; j < min(items, it + NS); j++) mbar_wait_bounded(bar0 + 8 * (j % NS), (uint32_t)((j / NS) & 1));
  };
  const int p0 = 16 * warp;  // this warp's block in every stage
  // ---- pass 1: scores ----
  for (int it = 0; it < nsub; it++) {
    const int st = it % NS;
    if (!__all_sync(0xFFFFFFFFu, mbar_wait_bounded(bar0 + 8 * st, (uint32_t)((it / NS) & 1)))) ok = false;
    const int rb = it * AT_SUB;
    const int np = min(AT_SUB, n - rb);
    if (ok && p0 < np) {
      const int m = lane >> 3, r = p0 + (lane & 7) + 8 * (m & 1), cadd = m >> 1;
      const uint32_t rowaddr = smem_u32(ring + st * AT_STAGE + r * 256);
      const int key = (t0 + rb + r) & 7;
      float acc[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; nt++) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < 8; ks++) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(rowaddr + (uint32_t)(((2 * ks + cadd) ^ key) << 4), a0, a1, a2, a3);
#pragma unroll
        for (int nt = 0; nt < NT; nt++) mma16816(acc[nt], a0, a1, a2, a3, qb[nt][ks][0], qb[nt][ks][1]);
      }
#pragma unroll
      for (int nt = 0; nt < NT; nt++) {
        const int h = 4 * nt + t;
        if (h < G) {
          const float f = qsc[h];
          if (p0 + g < np) sc[h * cp + rb + p0 + g] = (acc[nt][0] + acc[nt][1]) * f;
          if (p0 + g + 8 < np) sc[h * cp + rb + p0 + g + 8] = (acc[nt][2] + acc[nt][3]) * f;
        }
      }
    }
    ok = !__syncthreads_or(!ok);  // stage consumed by every warp
    if (!ok) {
      drain(it);
      break;
    }
    if (tid == 0 && it + NS < items) issue(it + NS);
  }
  // ---- softmax statistics per head (TensorOps.Softmax: max, exp, sum) ----
  for (int h = warp; h < G && ok; h += AT_WARPS) {
    float m = -INFINITY;
    for (int i = lane; i < n; i += 32) m = fmaxf(m, sc[h * cp + i]);
    m = warp_max(m);
    float l = 0.f;
    uint16_t* ph = pp + (size_t)h * cp;
    uint16_t* pl = pp + (size_t)(G + h) * cp;
    for (int i = lane; i < nsub * AT_SUB; i += 32) {
      float p = 0.f;
      if (i < n) {
        p = expf(sc[h * cp + i] - m);
        l += p;
      }
      const __half hi = __float2half_rn(p);
      ph[i] = __half_as_ushort(hi);
      pl[i] = __half_as_ushort(__float2half_rn(p - __half2float(hi)));
    }
    l = warp_sum(l);
    if (lane == 0) {
      stat[2 * h] = n > 0 ? m : -INFINITY;
      stat[2 * h + 1] = l;
    }
  }
  __syncthreads();
  // ---- pass 2: o^T[d][h] = sum_t V_t[d] p[h][t] ----
  float o[NT][8][4];
#pragma unroll
  for (int nt = 0; nt < NT; nt++)
#pragma unroll
    for (int mt = 0; mt < 8; mt++) o[nt][mt][0] = o[nt][mt][1] = o[nt][mt][2] = o[nt][mt][3] = 0.f;
  for (int it = nsub; it < items && ok; it++) {
    const int st = it % NS;
    if (!__all_sync(0xFFFFFFFFu, mbar_wait_bounded(bar0 + 8 * st, (uint32_t)((it / NS) & 1)))) ok = false;
    const int rb = (it - nsub) * AT_SUB;
    const int np = min(AT_SUB, n - rb);
    uint8_t* vst = ring + st * AT_STAGE;
    if (ok && p0 < np) {
      if (np - p0 < 16) {  // rows past the chunk: zero them (their p is 0, 0 * stale could be NaN)
        uint4* z = (uint4*)(vst + np * 256);
        for (int i = lane; i < (p0 + 16 - np) * 16; i += 32) z[i] = make_uint4(0u, 0u, 0u, 0u);
        __syncwarp();
      }
      uint32_t pb[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; nt++) {
        const int h = 4 * nt + (g >> 1), part = g & 1;
        if (h < G) {
          const uint16_t* pr = pp + (size_t)(part * G + h) * cp + rb + p0 + 2 * t;
          pb[nt][0] = *(const uint32_t*)pr;
          pb[nt][1] = *(const uint32_t*)(pr + 8);
        } else {
          pb[nt][0] = pb[nt][1] = 0u;
        }
      }
      const int m = lane >> 3, r = p0 + (lane & 7) + 8 * (m >> 1), cadd = m & 1;
      const uint32_t rowaddr = smem_u32(vst + r * 256);
      const int key = (t0 + rb + r) & 7;
#pragma unroll
      for (int mt = 0; mt < 8; mt++) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4_t(rowaddr + (uint32_t)(((2 * mt + cadd) ^ key) << 4), a0, a1, a2, a3);
#pragma unroll
        for (int nt = 0; nt < NT; nt++) mma16816(o[nt][mt], a0, a1, a2, a3, pb[nt][0], pb[nt][1]);
      }
    }
    ok = !__syncthreads_or(!ok);
    if (!ok) {
      drain(it);
      break;
    }
    if (tid == 0 && it + NS < items) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // zeroed rows before the refill
      issue(it + NS);
    }
  }
  // reduce the warps' partial outputs
#pragma unroll
  for (int nt = 0; nt < NT; nt++) {
    const int h = 4 * nt + t;
    if (h < G) {
#pragma unroll
      for (int mt = 0; mt < 8; mt++) {
        ored[(warp * G + h) * HD + 16 * mt + g] = o[nt][mt][0] + o[nt][mt][1];
        ored[(warp * G + h) * HD + 16 * mt + g + 8] = o[nt][mt][2] + o[nt][mt][3];
      }
    }
  }
  __syncthreads();
  const int64_t pbase = (((int64_t)b * a.nh + kvh * G) * S + s_idx);  // head h: + h*S
  for (int i = tid; i < G * HD; i += blockDim.x) {
    const int h = i / HD, d = i % HD;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < AT_WARPS; w++) v += ored[(w * G + h) * HD + d];
    a.part_o[(pbase + (int64_t)h * S) * HD + d] = v;
  }
  if (tid < G) {
    a.part_ml[(pbase + (int64_t)tid * S) * 2 + 0] = stat[2 * tid];
    a.part_ml[(pbase + (int64_t)tid * S) * 2 + 1] = stat[2 * tid + 1];
  }
  if (!ok && tid == 0) atomicOr(a.err, SI_DEVERR_WAIT_TIMEOUT);
  if (G >= 2 && a.merge_cnt) attn_merge_last<G>(a, smem, b, kvh, S);
}

}  // namespace

size_t attn_smem_bytes(int G, int chunk_max, int ns) {
  const AttnSmem L{G, (chunk_max + 63) & ~63, ns};
  return L.total();
}

int launch_attn(cudaStream_t s, const AttnArgs& a, int G, int splits, int batch, int nkv, bool pdl) {
  const int ns = batch >= 4 ? 2 : AT_NS;
  const size_t smem = attn_smem_bytes(G, a.chunk_max, ns);
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
    if (ns == 2) {                                                                            \
      SI_CUDA(cudaFuncSetAttribute(k_attn_decode<GG, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                   (int)smem));                                               \
      SI_CUDA(cudaLaunchKernelEx(&cfg, k_attn_decode<GG, 2>, a));                             \
    } else {                                                                                  \
      SI_CUDA(cudaFuncSetAttribute(k_attn_decode<GG, AT_NS>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                   (int)smem));                                               \
      SI_CUDA(cudaLaunchKernelEx(&cfg, k_attn_decode<GG, AT_NS>, a));                         \
    }                                                                                         \
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
