// Model-level prefill: the n prompt tokens of one sequence through every
// layer at once, on the tensor cores, filling the f16 KV cache.  This
// replaces the reference's prefill loop, one Transformer.Forward per prompt
// token (src/SharpInfer.Core/Engine/InferenceEngine.cs:82-85), with one GEMM
// per projection and one causal flash-attention per layer
// (FlashAttention.Forward, src/SharpInfer.Core/Layers/FlashAttention.cs:59-167).
//
// Per layer (rows = the n tokens):
//   k_rms_rows       RmsNorm(x) * attn_norm -> f16 rows, each scaled by a power
//                    of two (the GEMM undoes it)                     (Transformer.cs:86)
//   GEMM             [Wq; Wk; Wv] -> qkv f32                         (:89-91)
//   k_rope_store     RoPE of q and k; k, v rounded to f16 into the cache at
//                    positions pos0 .. pos0 + n - 1 (KVCache.Store); q to f16
//                    [head][row][128]                                 (:94-97)
//   k_cache_dense    cache positions 0 .. pos0 + n - 1 -> dense f16 K, V
//   attention        causal, start_pos = pos0, on the cache's f16 values (:99-129)
//   k_heads_rows     o [head][row][128] -> f16 rows [row][head * 128]
//   GEMM             Wo, added to x                                    (:132-135)
//   k_rms_rows       RmsNorm(x) * ffn_norm                             (:140)
//   GEMM             [Wgate; Wup] -> gu f32                            (:143-144)
//   k_silu_rows      SiLU(gate) * up -> f16 rows                       (:147-148)
//   GEMM             Wdown, added to x                                 (:151-154)
// The stored K/V are those the decode step would store token by token (same
// RoPE table and arithmetic, same f16 rounding); the activations enter the
// GEMMs as f16 (11 significant bits after the per-row power-of-two scale).
#include "model.cuh"
#include "quantfmt.cuh"

namespace si {
namespace {

constexpr int HD = 128;

// Largest |v| of a block's values (each thread passes its own maximum).
__device__ __forceinline__ float block_amax(float m, float* red) {
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); i++) t = fmaxf(t, red[i]);
  __syncthreads();
  return t;
}

// Power-of-two scale that puts the largest |v| of a row in [2^14, 2^15).
__device__ __forceinline__ int row_exponent(float amax) {
  int e = 0;
  if (amax > 0.f && amax <= 3.0e38f) {
    int E;
    frexpf(amax, &E);  // amax < 2^E
    e = 15 - E;
    e = e < -100 ? -100 : (e > 100 ? 100 : e);
  }
  return e;
}

// x[i] = row tokens[i] of the token embedding (Transformer.cs:76).
__global__ void k_embed_rows(const int* __restrict__ tokens, int qt, const uint8_t* __restrict__ W, int64_t nblk,
                             int64_t vocab, int h, float* __restrict__ x) {
  const int i = blockIdx.y, col = blockIdx.x * blockDim.x + threadIdx.x;
  const int tok = tokens[i];
  if (col < h && tok >= 0 && tok < vocab) x[(int64_t)i * h + col] = dev_weight_elem(qt, W, nblk, tok, col);
}

// Row i: v = (x * scale) * w with scale = 1 / sqrtf(sum x^2 / h + eps)
// (TensorOps.RmsNorm, TensorOps.cs:135-145), stored as f16(v 2^e), rs = 2^-e.
// One CTA per row; v kept in shared memory (h <= 16384).
__global__ void __launch_bounds__(256) k_rms_rows(const float* __restrict__ x, int h, const float* __restrict__ w,
                                                  float eps, __half* __restrict__ y, float* __restrict__ rs) {
  extern __shared__ float sv[];
  __shared__ float red[8];
  const int i = blockIdx.x, tid = threadIdx.x;
  const float* xr = x + (int64_t)i * h;
  float ss = 0.f;
  for (int k = tid; k < h; k += 256) {
    const float v = xr[k];
    sv[k] = v;
    ss = __fadd_rn(ss, __fmul_rn(v, v));
  }
  ss = warp_sum(ss);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float t = 0.f;
  for (int k = 0; k < 8; k++) t += red[k];
  __syncthreads();
  const float scale = 1.0f / sqrtf(t / (float)h + eps);
  float m = 0.f;
  for (int k = tid; k < h; k += 256) {
    const float v = __fmul_rn(__fmul_rn(sv[k], scale), w[k]);
    sv[k] = v;
    m = fmaxf(m, fabsf(v));
  }
  const int e = row_exponent(block_amax(m, red));
  const float s = ldexpf(1.0f, e);
  for (int k = tid; k < h; k += 256) y[(int64_t)i * h + k] = __float2half_rn(sv[k] * s);
  if (tid == 0) rs[i] = ldexpf(1.0f, -e);
}

// RoPE (RotaryEmbedding.ApplyToHead: adjacent pairs, angles from the host
// table) of row i's q and k heads; k and v rounded to f16 into the cache at
// position pos0 + i (KVCache.Store), q to f16 qh [head][row][128].
// Grid (n rows, nh + nkv head slots), 64 threads: one pair of dims each.
__global__ void k_rope_store(const float* __restrict__ qkv, int ld, const float* __restrict__ rope, int pos0, int n,
                             int nh, int nkv, __half* __restrict__ kc, __half* __restrict__ vc, int max_seq,
                             __half* __restrict__ qh) {
  const int i = blockIdx.x, slot = blockIdx.y, p = threadIdx.x;
  const int pos = pos0 + i;
  const float* row = qkv + (int64_t)i * ld;
  const float2 cs = ((const float2*)(rope + (int64_t)pos * HD))[p];
  if (slot < nh) {
    const float* q = row + (int64_t)slot * HD;
    const float x0 = q[2 * p], x1 = q[2 * p + 1];
    const float r0 = __fsub_rn(__fmul_rn(x0, cs.x), __fmul_rn(x1, cs.y));
    const float r1 = __fadd_rn(__fmul_rn(x0, cs.y), __fmul_rn(x1, cs.x));
    *(__half2*)(qh + ((int64_t)slot * n + i) * HD + 2 * p) = __halves2half2(__float2half_rn(r0), __float2half_rn(r1));
  } else {
    const int kvh = slot - nh;
    const float* k = row + (int64_t)(nh + kvh) * HD;
    const float* v = row + (int64_t)(nh + nkv + kvh) * HD;
    const float x0 = k[2 * p], x1 = k[2 * p + 1];
    const float r0 = __fsub_rn(__fmul_rn(x0, cs.x), __fmul_rn(x1, cs.y));
    const float r1 = __fadd_rn(__fmul_rn(x0, cs.y), __fmul_rn(x1, cs.x));
    const int64_t o = ((int64_t)kvh * max_seq + pos) * HD + kv_swz(2 * p, pos);
    *(__half2*)(kc + o) = __halves2half2(__float2half_rn(r0), __float2half_rn(r1));
    *(__half2*)(vc + o) = __halves2half2(__float2half_rn(v[2 * p]), __float2half_rn(v[2 * p + 1]));
  }
}

// Cache positions [0, len) of every kv head -> dense [nkv][len][128] (the
// 16-byte chunks put back in order).  One thread per 16-byte chunk.
__global__ void k_cache_dense(const __half* __restrict__ cache, int max_seq, int len, int nkv,
                              __half* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)nkv * len * 16) return;
  const int c = (int)(i & 15);
  const int64_t pr = i >> 4;  // kvh * len + pos
  const int pos = (int)(pr % len), kvh = (int)(pr / len);
  const uint4* src = (const uint4*)(cache + ((int64_t)kvh * max_seq + pos) * HD);
  ((uint4*)out)[i] = src[c ^ (pos & 7)];
}

// o [head][row][128] f32 -> row i of f16 [row][nh * 128], scaled by 2^e.
__global__ void __launch_bounds__(256) k_heads_rows(const float* __restrict__ o, int n, int nh,
                                                    __half* __restrict__ y, float* __restrict__ rs) {
  __shared__ float red[8];
  const int i = blockIdx.x, tid = threadIdx.x, K = nh * HD;
  float m = 0.f;
  for (int k = tid; k < K; k += 256) m = fmaxf(m, fabsf(o[((int64_t)(k >> 7) * n + i) * HD + (k & 127)]));
  const int e = row_exponent(block_amax(m, red));
  const float s = ldexpf(1.0f, e);
  for (int k = tid; k < K; k += 256)
    y[(int64_t)i * K + k] = __float2half_rn(o[((int64_t)(k >> 7) * n + i) * HD + (k & 127)] * s);
  if (tid == 0) rs[i] = ldexpf(1.0f, -e);
}

// Row i: v = SiLU(gate) * up (TensorOps.SiLU then MulInPlace, the decode
// step's arithmetic) from gu [row][2 inter] -> f16 [row][inter], scaled by 2^e.
__device__ __forceinline__ float silu_mul(float g, float u) {
  return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
}
__global__ void __launch_bounds__(256) k_silu_rows(const float* __restrict__ gu, int inter, __half* __restrict__ y,
                                                   float* __restrict__ rs) {
  __shared__ float red[8];
  const int i = blockIdx.x, tid = threadIdx.x;
  const float* g = gu + (int64_t)i * 2 * inter;
  float m = 0.f;
  for (int k = tid; k < inter; k += 256) m = fmaxf(m, fabsf(silu_mul(g[k], g[inter + k])));
  const int e = row_exponent(block_amax(m, red));
  const float s = ldexpf(1.0f, e);
  for (int k = tid; k < inter; k += 256) y[(int64_t)i * inter + k] = __float2half_rn(silu_mul(g[k], g[inter + k]) * s);
  if (tid == 0) rs[i] = ldexpf(1.0f, -e);
}

}  // namespace

int launch_embed_rows(cudaStream_t s, const int* tokens, int n, const si_weight* emb, int h, float* x) {
  k_embed_rows<<<dim3((unsigned)((h + 255) / 256), (unsigned)n), 256, 0, s>>>(tokens, emb->qtype,
                                                                            (const uint8_t*)emb->dev, emb->nblk,
                                                                            emb->rows, h, x);
  SI_CUDA(cudaGetLastError());
  return SI_OK;
}

int launch_rms_rows(cudaStream_t s, const float* x, int n, int h, const float* w, float eps, __half* y, float* rs) {
  const size_t smem = (size_t)h * 4;
  if (smem > 64 * 1024) {
    static DeviceOnce attr;
    int dev = 0;
    SI_CUDA(cudaGetDevice(&dev));
    if (!attr.done(dev)) {
      SI_CUDA(cudaFuncSetAttribute(k_rms_rows, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
      attr.mark(dev);
    }
  }
  if (smem > 200 * 1024) SI_FAIL(SI_ERR_UNSUPPORTED, "prefill: hidden size %d too large", h);
  k_rms_rows<<<(unsigned)n, 256, smem, s>>>(x, h, w, eps, y, rs);
  SI_CUDA(cudaGetLastError());
  return SI_OK;
}

int launch_rope_store(cudaStream_t s, const float* qkv, int ld, const float* rope, int pos0, int n, int nh, int nkv,
                      __half* kc, __half* vc, int max_seq, __half* qh) {
  k_rope_store<<<dim3((unsigned)n, (unsigned)(nh + nkv)), HD / 2, 0, s>>>(qkv, ld, rope, pos0, n, nh, nkv, kc, vc,
                                                                         max_seq, qh);
  SI_CUDA(cudaGetLastError());
  return SI_OK;
}

int launch_cache_dense(cudaStream_t s, const __half* cache, int max_seq, int len, int nkv, __half* out) {
  const int64_t chunks = (int64_t)nkv * len * 16;
  k_cache_dense<<<(unsigned)((chunks + 255) / 256), 256, 0, s>>>(cache, max_seq, len, nkv, out);
  SI_CUDA(cudaGetLastError());
  return SI_OK;
}

int launch_heads_rows(cudaStream_t s, const float* o, int n, int nh, __half* y, float* rs) {
  k_heads_rows<<<(unsigned)n, 256, 0, s>>>(o, n, nh, y, rs);
  SI_CUDA(cudaGetLastError());
  return SI_OK;
}

int launch_silu_rows(cudaStream_t s, const float* gu, int n, int inter, __half* y, float* rs) {
  k_silu_rows<<<(unsigned)n, 256, 0, s>>>(gu, inter, y, rs);
  SI_CUDA(cudaGetLastError());
  return SI_OK;
}

}  // namespace si
