// Decode-model internals shared by model.cu and attn.cu.
#pragma once
#include "common.cuh"

namespace si {

// Per-step parameters, copied from pinned host memory at the start of each
// decode-step graph.
struct StepParams {
  int pos;
  int batch;
  int tokens[SI_MAX_BATCH];
  int step;      // steps taken since the parameters were last written by the host
  int hist_cap;  // steps the history buffer holds
  int* hist;     // [hist_cap][batch] greedy tokens of consecutive steps
  unsigned epoch;  // steps since the model was created (tensor-parallel flag values)
};

struct AttnArgs {
  const StepParams* params;
  int layer, max_batch, max_seq, nh;
  __half* kcache;
  __half* vcache;
  const float* qkv;
  int64_t qkv_ld;
  const float* rope;  // [max_seq][head_dim/2][2] cos, sin
  float scale;        // 1 / sqrtf(head_dim)
  int chunk_max;      // positions per split at the longest context
  float* part_o;      // [batch][nh][splits][head_dim]
  float* part_ml;     // [batch][nh][splits][2]
  int* err;
  // Merge in the kernel (G >= 2): the last CTA of each (sequence, kv head) to
  // finish merges the splits of its G heads and packs them as prepared
  // O-projection input.  merge_cnt [max_batch][kv heads] counts finished
  // CTAs (zero between launches; the merging CTA resets it).
  int* merge_cnt = nullptr;
  uint8_t* xprep = nullptr;  // prepared-activation buffer of the O projection
  float* out = nullptr;      // optional f32 copy of the merged output [batch][nh * head_dim]
  L2Prefetch pf;             // a later kernel's weights, prefetched into L2 at launch
};

// KV cache rows are 128 f16 (256 B).  The 16-byte chunk c (dims 8c..8c+7) of
// position p is stored at chunk c ^ (p & 7), so that eight consecutive
// positions read at one chunk index hit eight different bank groups
// (ldmatrix without conflicts).  Offset in halves of dim d of position p:
__host__ __device__ __forceinline__ int kv_swz(int d, int p) { return (((d >> 3) ^ (p & 7)) << 3) | (d & 7); }

// Model-level prefill kernels (prefill.cu).
int launch_embed_rows(cudaStream_t s, const int* tokens, int n, const si_weight* emb, int h, float* x);
int launch_rms_rows(cudaStream_t s, const float* x, int n, int h, const float* w, float eps, __half* y, float* rs);
int launch_rope_store(cudaStream_t s, const float* qkv, int ld, const float* rope, int pos0, int n, int nh, int nkv,
                      __half* kc, __half* vc, int max_seq, __half* qh);
int launch_cache_dense(cudaStream_t s, const __half* cache, int max_seq, int len, int nkv, __half* out);
int launch_heads_rows(cudaStream_t s, const float* o, int n, int nh, __half* y, float* rs);
int launch_silu_rows(cudaStream_t s, const float* gu, int n, int inter, __half* y, float* rs);

size_t attn_smem_bytes(int G, int chunk_max, int ns);
int launch_attn(cudaStream_t s, const AttnArgs& a, int G, int splits, int batch, int nkv, bool pdl);

}  // namespace si
