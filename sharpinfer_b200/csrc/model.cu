// Decode model: weights, f16 KV cache, and the decode step of
// Transformer.Forward (src/SharpInfer.Core/Layers/Transformer.cs:67-162) as a
// sequence of fused kernels, captured once per batch size as a CUDA graph.
//
// Per layer (batch B, position pos):
//   prep   RmsNorm(x) * attn_norm -> activation fragments        (:86)
//   qmv    [Wq; Wk; Wv] -> qkv                                    (:89-91)
//   attn   RoPE(q, k), KV append, split-KV attention -> partials   (:94-129)
//   prep   merge of the splits -> fragments
//   qmv    Wo, accumulated into x (the residual add)              (:132-135)
//   prep   RmsNorm(x) * ffn_norm                                  (:140)
//   qmv    [Wgate; Wup] -> gu                                     (:143-144)
//   prep   SiLU(gate) * up                                        (:147-148)
//   qmv    Wdown, accumulated into x                              (:151-154)
// then RmsNorm(x) * final_norm, lm_head -> logits, ArgMax.         (:158-159)
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <map>
#include <vector>

#include "model.cuh"
#include "quantfmt.cuh"
#include "synth.h"

namespace si {
namespace {

// x[b] = row tokens[b] of the token embedding (Transformer.cs:76).
__global__ void k_embed(const StepParams* __restrict__ p, int qt, const uint8_t* __restrict__ W,
                        int64_t nblk, int64_t vocab, int h, float* __restrict__ x) {
  pdl_launch();  // dependents may start their independent prologue now
  pdl_wait();
  const int b = blockIdx.y;
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  const int tok = p->tokens[b];
  if (col < h && tok >= 0 && tok < vocab) x[(int64_t)b * h + col] = dev_weight_elem(qt, W, nblk, tok, col);
}

// Greedy selection (SamplingPipeline.ArgMax, SamplingPipeline.cs:83-89):
// first index of the maximum under strict '>'; NaNs never win, and a NaN at
// index 0 makes the answer 0.
// Tensor parallelism: each rank holds the vocabulary slice [rank * vocab, (rank +
// 1) * vocab); its candidate (value, global index) goes to every rank, and
// every rank takes the largest value, ties to the lowest index.  A NaN at
// global index 0 still makes the answer 0 (it is sent as +inf at index 0).
struct ArgmaxTp {
  uint8_t* const* peers = nullptr;
  const uint8_t* comm = nullptr;
  const unsigned* epoch = nullptr;
  int* err = nullptr;
  int tp = 1, rank = 0;
};

__global__ void __launch_bounds__(1024) k_argmax(const float* __restrict__ logits, int64_t vocab,
                                                 int* __restrict__ out, ArgmaxTp tp) {
  __shared__ float sv[32];
  __shared__ int si[32];
  pdl_launch();  // dependents may start their independent prologue now
  pdl_wait();
  const int b = blockIdx.x;
  const float* x = logits + (int64_t)b * vocab;
  float bv = -INFINITY;
  int bi = -1;
  auto consider = [&](float v, int i) {
    if (v > bv || (bi < 0 && v == bv)) {  // -inf candidates still record an index
      bv = v;
      bi = i;
    }
  };
  // Each thread visits its indices in increasing order: 16-byte loads, eight
  // in flight, then the scalar tail.
  const int nt = blockDim.x;
  const int n4 = (vocab % 4 == 0 && ((uintptr_t)x & 15) == 0) ? (int)(vocab / 4) : 0;
  for (int j0 = threadIdx.x; j0 < n4; j0 += 8 * nt) {
    float4 r[8];
#pragma unroll
    for (int u = 0; u < 8; u++) {
      const int j = j0 + u * nt;
      r[u] = j < n4 ? __ldcg((const float4*)x + j) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < 8; u++) {
      const int j = j0 + u * nt;
      if (j < n4) {
        consider(r[u].x, 4 * j);
        consider(r[u].y, 4 * j + 1);
        consider(r[u].z, 4 * j + 2);
        consider(r[u].w, 4 * j + 3);
      }
    }
  }
  for (int i = 4 * n4 + threadIdx.x; i < (int)vocab; i += nt) consider(x[i], i);
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
    const int oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
    if (oi >= 0 && (bi < 0 || ov > bv || (ov == bv && oi < bi))) {
      bv = ov;
      bi = oi;
    }
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) {
    sv[w] = bv;
    si[w] = bi;
  }
  __syncthreads();
  if (w == 0) {
    bv = l < (int)(blockDim.x >> 5) ? sv[l] : -INFINITY;
    bi = l < (int)(blockDim.x >> 5) ? si[l] : -1;
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
      const int oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
      if (oi >= 0 && (bi < 0 || ov > bv || (ov == bv && oi < bi))) {
        bv = ov;
        bi = oi;
      }
    }
    if (l == 0) {
      if (tp.tp == 1) {
        out[b] = (isnan(x[0]) || bi < 0) ? 0 : bi;
      } else {
        float cv = bi < 0 ? -INFINITY : bv;
        int ci = bi < 0 ? 0 : bi + tp.rank * (int)vocab;
        if (tp.rank == 0 && isnan(x[0])) {
          cv = INFINITY;
          ci = 0;
        }
        const unsigned want = *tp.epoch + 1u;
        for (int p = 0; p < tp.tp; p++) {
          uint2* slot = (uint2*)(tp.peers[p] + SI_TP_ARGMAX) + (b * SI_TP_MAX + tp.rank) * 2;
          st_tagged(slot, __float_as_uint(cv), want);
          st_tagged(slot + 1, (uint32_t)ci, want);
        }
        float gv = -INFINITY;
        int gi = -1;
        for (int r = 0; r < tp.tp; r++) {
          const uint2* c = (const uint2*)(tp.comm + SI_TP_ARGMAX) + (b * SI_TP_MAX + r) * 2;
          const float v = __uint_as_float(wait_tagged(c, want, tp.err));
          const int idx = (int)wait_tagged(c + 1, want, tp.err);
          if (gi < 0 || v > gv || (v == gv && idx < gi)) {
            gv = v;
            gi = idx;
          }
        }
        out[b] = gi < 0 ? 0 : gi;
      }
    }
  }
}

// End of a step: the greedy tokens become the next step's inputs at the next
// position (the decode loop of InferenceEngine.GenerateAsync,
// InferenceEngine.cs:96-131, with greedy sampling) and are appended to the
// history.
__global__ void k_advance(StepParams* __restrict__ p, const int* __restrict__ argmax) {
  pdl_launch();  // dependents may start their independent prologue now
  pdl_wait();
  const int b = threadIdx.x;
  const int B = p->batch;
  __syncthreads();
  if (b < B) {
    const int t = argmax[b];
    if (p->hist && p->step < p->hist_cap) p->hist[(int64_t)p->step * B + b] = t;
    p->tokens[b] = t;
  }
  __syncthreads();
  if (b == 0) {
    p->pos += 1;
    p->step += 1;
    p->epoch += 1;
  }
}

// Seeded f16 N(0,1) for positions [0, len) of one (layer, seq) cache; the
// generator index follows the reference layout [pos][kv head][dim].
// (With tensor parallelism this rank holds kv heads kvh0 .. kvh0 + nkv - 1 of nkv_g.)
__global__ void k_kv_synth(__half* __restrict__ cache, uint64_t key, int len, int nkv, int max_seq, int nkv_g,
                           int kvh0) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t n = (int64_t)len * nkv * 128;
  if (i >= n) return;
  const int d = (int)(i % 128), kvh = (int)((i / 128) % nkv);
  const int64_t pos = i / (128 * nkv);
  const int64_t gi = (pos * nkv_g + kvh0 + kvh) * 128 + d;
  cache[((int64_t)kvh * max_seq + pos) * 128 + kv_swz(d, (int)pos)] =
      __ushort_as_half(si_synth_f16(key, (uint64_t)gi, 1.0f));
}

__global__ void k_f32_synth(float* __restrict__ out, uint64_t key, int64_t n, float mean, float sigma) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = si_synth_f32(key, (uint64_t)i, mean, sigma);
}

// [n][nkv][128] (reference layout) -> [nkv][max_seq][128] at pos0.
__global__ void k_kv_scatter(__half* __restrict__ cache, const uint16_t* __restrict__ src, int pos0,
                             int n, int nkv, int max_seq, int nkv_g, int kvh0) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)n * nkv * 128) return;
  const int d = (int)(i % 128), kvh = (int)((i / 128) % nkv);
  const int64_t t = i / (128 * nkv);
  cache[((int64_t)kvh * max_seq + pos0 + t) * 128 + kv_swz(d, (int)(pos0 + t))] =
      __ushort_as_half(src[(t * nkv_g + kvh0 + kvh) * 128 + d]);
}

cudaLaunchConfig_t cfg_of(cudaStream_t s, dim3 g, dim3 b, size_t smem, bool pdl, cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = g;
  cfg.blockDim = b;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cfg;
}

float recipe_sigma(int qt, int recipe, int64_t cols) {
  const float rc = sqrtf((float)cols);
  if (qt == SI_Q4_K) return recipe == SI_SYNTH_MODEL ? 1.0f / (23.3f * rc) : 0.01f;
  if (qt == SI_Q6_K) return 1.0f / (348.0f * rc);
  return 1.0f / (73.9f * rc);  // Q8_0: rms of a uniform int8 is ~73.9
}

// Layout choices of the decode step (all give the same results):
//   SI_PLAN_MERGE_IN_ATTN  the last attention CTA of each kv head merges the
//                          splits and packs the O projection's input (G >= 2)
//                          instead of a separate merge kernel
//   SI_PLAN_SILU_IN_DOWN   the batch-1 down-projection matvec computes
//                          SiLU(gate) * up itself instead of a separate kernel
//   SI_PLAN_L2_PREFETCH    each kernel pulls the weights of the kernel two
//                          launches later into L2
//   SI_PLAN_FULL_RING      each batch-1 matvec CTA requests its whole
//                          shared-memory ring before waiting for its input
//   SI_PLAN_SELF_PREFETCH  each batch-1 matvec CTA pulls its own weights into
//                          L2 at launch and fills its shared-memory ring once
//                          its input is prepared
//   SI_PLAN_Q1_8WARPS      batch-1 matvec CTAs of 8 warps instead of 16, so a
//                          CTA of the following kernel fits beside one
//   SI_PLAN_TP_PREP_APART  tensor parallel, batch 1: the residual + partial
//                          sums and RmsNorm in a k_prep launch of their own
//                          instead of inside the qkv / gate-up matvec
enum : unsigned {
  SI_PLAN_MERGE_IN_ATTN = 1, SI_PLAN_SILU_IN_DOWN = 2, SI_PLAN_L2_PREFETCH = 4, SI_PLAN_SELF_PREFETCH = 8,
  SI_PLAN_Q1_8WARPS = 16, SI_PLAN_FULL_RING = 32, SI_PLAN_TP_PREP_APART = 64
};
constexpr unsigned SI_PLAN_DEFAULT = 0;

// The plan: SHARPINFER_B200_STEP_PLAN (a comma-separated subset of "merge",
// "silu", "prefetch", "selfprefetch", "w8", "fullring", "tpapart", or
// "none") when set, else SI_PLAN_DEFAULT.
unsigned step_plan() {
  const char* e = getenv("SHARPINFER_B200_STEP_PLAN");
  if (!e) return SI_PLAN_DEFAULT;
  unsigned p = 0;
  if (strstr(e, "merge")) p |= SI_PLAN_MERGE_IN_ATTN;
  if (strstr(e, "silu")) p |= SI_PLAN_SILU_IN_DOWN;
  if (strstr(e, "prefetch") && !strstr(e, "selfprefetch")) p |= SI_PLAN_L2_PREFETCH;
  if (strstr(e, "selfprefetch")) p |= SI_PLAN_SELF_PREFETCH;
  if (strstr(e, "w8")) p |= SI_PLAN_Q1_8WARPS;
  if (strstr(e, "fullring")) p |= SI_PLAN_FULL_RING;
  if (strstr(e, "tpapart")) p |= SI_PLAN_TP_PREP_APART;
  return p;
}

L2Prefetch pf_of(const si_weight* w) {
  L2Prefetch p;
  if (w && w->bytes < (1ull << 32)) {
    p.ptr = (const uint8_t*)w->dev;
    p.bytes = (uint32_t)(w->bytes & ~(size_t)15);
  }
  return p;
}

}  // namespace
}  // namespace si

using namespace si;

struct si_model {
  si_ctx* c = nullptr;
  si_model_config cfg{};   // this rank's shapes (heads, kv heads, FFN rows, vocabulary slice)
  si_model_config gcfg{};  // the whole model's shapes
  int tp = 1, rank = 0;    // tensor parallelism
  uint8_t* comm = nullptr;                 // this rank's communication buffer (tp > 1)
  uint8_t* peer_base[SI_TP_MAX] = {};      // every rank's buffer mapped here
  uint8_t** peers_dev = nullptr;           // the same table on the device
  bool connected = false;
  bool ipc = false;                        // peers mapped through CUDA IPC (closed on free)
  unsigned epoch = 0;                      // steps taken (mirrors StepParams::epoch)
  int G = 0, qkv_rows = 0, Kmax = 0;
  int splits_max = 0, chunk_max = 0;
  std::vector<si_weight*> wqkv, wo, wgu, wdown;
  si_weight* emb = nullptr;
  si_weight* lm_head = nullptr;
  float* norms = nullptr;  // [L][2][h], then final [h]
  __half* kcache = nullptr;
  __half* vcache = nullptr;
  float* rope = nullptr;
  float *x = nullptr, *x2 = nullptr, *qkv = nullptr, *gu = nullptr, *logits = nullptr;
  int* argmax = nullptr;
  uint8_t* xprep = nullptr;
  float *part_o = nullptr, *part_ml = nullptr;
  int* merge_cnt = nullptr;  // [max_batch][kv heads] CTAs of the attention kernel done (merge in the kernel)
  unsigned plan = 0;         // SI_PLAN_* bits: how the decode step is laid out
  StepParams* dparams = nullptr;
  StepParams* hparams = nullptr;  // pinned
  int* hargmax = nullptr;         // pinned
  int* hist = nullptr;            // device token history of si_decode_generate
  int64_t hist_cap = 0;           // ints
  // model-level prefill scratch (grow-only, allocated on first use)
  si_devbuf pf_tok, pf_x, pf_xh, pf_rs, pf_qkv, pf_gu, pf_q, pf_k, pf_v, pf_o;
  std::map<int, cudaGraphExec_t> graphs;
  std::map<int, int> graph_kernels;  // kernel launches per captured step
  std::vector<void*> allocs;
};

namespace {

int dev_alloc(si_model* m, void** p, size_t bytes) {
  cudaError_t e = cudaMalloc(p, bytes);
  if (e != cudaSuccess)
    SI_FAIL(e == cudaErrorMemoryAllocation ? SI_ERR_OOM : SI_ERR_CUDA, "model allocation of %zu bytes failed: %s",
            bytes, cudaGetErrorString(e));
  m->allocs.push_back(*p);
  return SI_OK;
}

int make_weight(si_model* m, int qt, int64_t rows, int64_t cols, si_weight** out) {
  si_weight* w = new si_weight();
  w->qtype = qt;
  w->rows = rows;
  w->cols = cols;
  w->tiles = (rows + 15) / 16;
  w->nblk = cols / block_elems(qt);
  w->bytes = (size_t)(w->tiles * w->nblk * tile_block_bytes(qt));
  w->device = m->c->device;
  cudaError_t e = cudaMalloc(&w->dev, w->bytes);
  if (e != cudaSuccess) {
    delete w;
    SI_FAIL(e == cudaErrorMemoryAllocation ? SI_ERR_OOM : SI_ERR_CUDA, "weight allocation failed: %s",
            cudaGetErrorString(e));
  }
  *out = w;
  return SI_OK;
}

// Which part of a whole tensor rank `rank` of `tp` holds: global rows grow0 ..
// grow0 + rows and, in each, quant blocks gb0 .. gb0 + nblk of gnblk.
// Column-parallel tensors (q, k, v, gate, up, lm_head) take a slice of rows,
// row-parallel ones (o, down) a slice of every row (Megatron layout); the
// embedding is replicated.
int tp_slice(const si_model_config& g, int tp, int rank, int t, int64_t* grow0, int64_t* rows, int64_t* gb0,
             int64_t* nblk, int64_t* gnblk) {
  const int64_t hd = g.head_dim;
  auto be = [](int qt) -> int64_t { return qt == SI_Q8_0 ? 32 : 256; };
  const int64_t bw = be(g.weight_qtype);
  auto colpar = [&](int64_t grows, int64_t cols, int qt) {
    *rows = grows / tp;
    *grow0 = (int64_t)rank * *rows;
    *gnblk = *nblk = cols / be(qt);
    *gb0 = 0;
  };
  auto rowpar = [&](int64_t grows, int64_t gcols) {
    *rows = grows;
    *grow0 = 0;
    *gnblk = gcols / bw;
    *nblk = *gnblk / tp;
    *gb0 = (int64_t)rank * *nblk;
  };
  switch (t) {
    case SI_T_Q: colpar((int64_t)g.n_heads * hd, g.hidden, g.weight_qtype); return SI_OK;
    case SI_T_K:
    case SI_T_V: colpar((int64_t)g.n_kv_heads * hd, g.hidden, g.weight_qtype); return SI_OK;
    case SI_T_GATE:
    case SI_T_UP: colpar(g.intermediate, g.hidden, g.weight_qtype); return SI_OK;
    case SI_T_O: rowpar(g.hidden, (int64_t)g.n_heads * hd); return SI_OK;
    case SI_T_DOWN: rowpar(g.hidden, g.intermediate); return SI_OK;
    case SI_T_LM_HEAD: colpar(g.vocab, g.hidden, g.lm_head_qtype); return SI_OK;
    case SI_T_EMB:
      *rows = g.vocab;
      *grow0 = *gb0 = 0;
      *gnblk = *nblk = g.hidden / be(g.emb_qtype);
      return SI_OK;
    default: SI_FAIL(SI_ERR_INVALID, "tensor %d is not a quantised tensor", t);
  }
}

// Where a tensor lives on this rank: the fused weight, the first local row
// inside it, and the part of the whole tensor (tp_slice) it holds.
struct Slot {
  si_weight* w;
  int64_t row0, rows;
  int64_t grow0, gnblk, gb0;
};

int tensor_slot(si_model* m, int layer, int t, Slot* sl) {
  const si_model_config& c = m->cfg;
  if ((layer < 0) != (t == SI_T_EMB || t == SI_T_LM_HEAD))
    SI_FAIL(SI_ERR_INVALID, "tensor %d with layer %d", t, layer);
  if (layer >= c.n_layers) SI_FAIL(SI_ERR_INVALID, "layer %d out of range", layer);
  int64_t grow0, rows, gb0, nblk, gnblk;
  SI_TRY(tp_slice(m->gcfg, m->tp, m->rank, t, &grow0, &rows, &gb0, &nblk, &gnblk));
  const int64_t qr = (int64_t)c.n_heads * c.head_dim, kr = (int64_t)c.n_kv_heads * c.head_dim;
  si_weight* w = nullptr;
  int64_t row0 = 0;
  switch (t) {
    case SI_T_Q: w = m->wqkv[layer]; break;
    case SI_T_K: w = m->wqkv[layer]; row0 = qr; break;
    case SI_T_V: w = m->wqkv[layer]; row0 = qr + kr; break;
    case SI_T_O: w = m->wo[layer]; break;
    case SI_T_GATE: w = m->wgu[layer]; break;
    case SI_T_UP: w = m->wgu[layer]; row0 = c.intermediate; break;
    case SI_T_DOWN: w = m->wdown[layer]; break;
    case SI_T_EMB: w = m->emb; break;
    case SI_T_LM_HEAD: w = m->lm_head; break;
    default: SI_FAIL(SI_ERR_INVALID, "tensor %d is not a quantised tensor", t);
  }
  if (w->nblk != nblk) SI_FAIL(SI_ERR_INVALID, "tensor %d: shard shape mismatch", t);
  *sl = Slot{w, row0, rows, grow0, gnblk, gb0};
  return SI_OK;
}

float* norm_ptr(si_model* m, int layer, int t) {
  const int64_t h = m->cfg.hidden;
  if (layer < 0) return m->norms + (int64_t)m->cfg.n_layers * 2 * h;
  return m->norms + ((int64_t)layer * 2 + (t == SI_T_FFN_NORM ? 1 : 0)) * h;
}

int check_config(const si_model_config* c) {
  if (!c) SI_FAIL(SI_ERR_INVALID, "model config is NULL");
  if (c->n_layers <= 0 || c->hidden <= 0 || c->intermediate <= 0 || c->vocab <= 0 || c->max_seq <= 0)
    SI_FAIL(SI_ERR_INVALID, "model config has non-positive sizes");
  if (c->head_dim != 128) SI_FAIL(SI_ERR_UNSUPPORTED, "head_dim %d (this build supports 128)", c->head_dim);
  if (c->n_heads <= 0 || c->n_kv_heads <= 0 || c->n_heads % c->n_kv_heads)
    SI_FAIL(SI_ERR_INVALID, "n_heads %d must be a positive multiple of n_kv_heads %d", c->n_heads, c->n_kv_heads);
  const int G = c->n_heads / c->n_kv_heads;
  if (G != 1 && G != 2 && G != 4 && G != 8) SI_FAIL(SI_ERR_UNSUPPORTED, "%d q heads per kv head", G);
  if (c->max_batch < 1 || c->max_batch > SI_MAX_BATCH) SI_FAIL(SI_ERR_INVALID, "max_batch %d outside 1..16", c->max_batch);
  // split-KV attention: at most 511 splits of at most 1024 positions (the last holds 16)
  if (c->max_seq > 510 * 1024) SI_FAIL(SI_ERR_UNSUPPORTED, "max_seq %d above %d", c->max_seq, 510 * 1024);
  for (int qt : {c->weight_qtype, c->lm_head_qtype, c->emb_qtype})
    if (qt != SI_Q4_K && qt != SI_Q6_K && qt != SI_Q8_0) SI_FAIL(SI_ERR_UNSUPPORTED, "quant type %d", qt);
  auto blk = [](int qt) { return qt == SI_Q8_0 ? 32 : 256; };
  if (c->hidden % blk(c->weight_qtype) || c->intermediate % blk(c->weight_qtype) ||
      (c->n_heads * c->head_dim) % blk(c->weight_qtype) || c->hidden % blk(c->lm_head_qtype) ||
      c->hidden % blk(c->emb_qtype))
    SI_FAIL(SI_ERR_INVALID, "hidden/intermediate must be multiples of the quant block size");
  if (c->hidden % 16 || c->intermediate % 16) SI_FAIL(SI_ERR_INVALID, "hidden and intermediate must be multiples of 16");
  if (c->hidden > SI_MAX_K || c->intermediate > SI_MAX_K) SI_FAIL(SI_ERR_UNSUPPORTED, "hidden/intermediate above %d", SI_MAX_K);
  return SI_OK;
}

// Splits of the attention kernel for batch B: enough CTAs for two per SM,
// and at most 1024 positions per split at the longest context -- 256 where
// the split count allows it, so that a CTA's scores fit beside a second CTA
// in shared memory (at batch 16 a 1024-position split leaves one 4-warp CTA
// per SM and the KV stream at a third of HBM bandwidth).
int attn_splits(const si_model* m, int B) {
  const int want = (2 * m->c->sm_count + B * m->cfg.n_kv_heads - 1) / (B * m->cfg.n_kv_heads);
  const int need = (m->cfg.max_seq + 1023) / 1024 + 1;  // the last split holds 16 positions
  const int fit = (m->cfg.max_seq + 255) / 256 + 1;
  return std::min(std::max(std::max(want, need), std::min(fit, m->splits_max)), m->splits_max);
}

int enqueue_attention(si_model* m, int layer, const float* qkv, float* out, int B, bool pdl,
                      L2Prefetch pf = L2Prefetch{}) {
  const si_model_config& c = m->cfg;
  AttnArgs a;
  a.params = m->dparams;
  a.layer = layer;
  a.max_batch = c.max_batch;
  a.max_seq = c.max_seq;
  a.nh = c.n_heads;
  a.kcache = m->kcache;
  a.vcache = m->vcache;
  a.qkv = qkv;
  a.qkv_ld = m->qkv_rows;
  a.rope = m->rope;
  a.scale = 1.0f / sqrtf((float)c.head_dim);  // Transformer.cs:101
  const int S = attn_splits(m, B);
  // all but the last split share the positions before the newest 16
  a.chunk_max = S > 1 ? (c.max_seq + S - 2) / (S - 1) : c.max_seq;
  a.part_o = m->part_o;
  a.part_ml = m->part_ml;
  a.err = m->c->dev_err;
  a.pf = pf;
  if (m->G >= 2 && (m->plan & SI_PLAN_MERGE_IN_ATTN)) {  // the last CTA of each kv head merges and packs
    a.merge_cnt = m->merge_cnt;
    a.xprep = m->xprep;
    a.out = out;
    return launch_attn(m->c->stream, a, m->G, S, B, c.n_kv_heads, pdl);
  }
  SI_TRY(launch_attn(m->c->stream, a, m->G, S, B, c.n_kv_heads, pdl));
  // one q head per kv head: a 256-column unit spans two kv heads, so a
  // separate kernel merges the splits into the prepared input (and `out`)
  return launch_prep(m->c->stream, m->part_o, S, m->part_ml, nullptr, 0.f, SI_PREP_ATTN_MERGE,
                     c.n_heads * c.head_dim, B, out, m->xprep, pdl);
}

// The whole decode step on the context stream (eager or under capture).
// Tensor-parallel arguments of the producer (kind 0: Wo, 1: Wdown of `layer`)
// and of its consumer, the RmsNorm prep that adds the partial sums.
QmvBuffers tp_producer(si_model* m, int layer, int kind) {
  QmvBuffers qb = m->c->qmv();
  qb.ring_mode = (m->plan & SI_PLAN_SELF_PREFETCH) ? 2 : (m->plan & SI_PLAN_FULL_RING) ? 1 : 0;
  qb.q1w = (m->plan & SI_PLAN_Q1_8WARPS) ? 8 : 16;
  const int64_t slot = (int64_t)m->cfg.max_batch * m->cfg.hidden * 8;
  qb.tp = TpArgs{m->peers_dev, &m->dparams->epoch, m->tp, m->rank, kind, 2 * layer + kind + 1,
                 2 * m->cfg.n_layers, SI_TP_SLOTS + (int64_t)kind * m->tp * slot + (int64_t)m->rank * slot,
                 m->cfg.hidden};
  return qb;
}
PrepTp tp_consumer(si_model* m, int layer, int kind) {
  const int64_t slot = (int64_t)m->cfg.max_batch * m->cfg.hidden * 8;
  PrepTp p;
  p.comm = m->comm;
  p.epoch = &m->dparams->epoch;
  p.err = m->c->dev_err;
  p.tp = m->tp;
  p.kind = kind;
  p.flag_add = 2 * layer + kind + 1;
  p.nlayers2 = 2 * m->cfg.n_layers;
  p.slots_off = SI_TP_SLOTS + (int64_t)kind * m->tp * slot;
  p.src_stride = slot;
  p.ld = m->cfg.hidden;
  return p;
}

// The whole decode step on the context stream (eager or under capture).  With
// tensor parallelism the Wo / Wdown matvecs store partial sums into every
// rank's slots and the following RmsNorm prep adds them to the residual,
// which alternates between x (before attention) and x2 (before the FFN).
int enqueue_step(si_model* m, int B) {
  const si_model_config& c = m->cfg;
  cudaStream_t s = m->c->stream;
  const int h = c.hidden, inter = c.intermediate, L = c.n_layers;
  const bool tp = m->tp > 1;
  const bool pre = (m->plan & SI_PLAN_L2_PREFETCH) != 0;
  QmvBuffers qb = m->c->qmv();
  qb.ring_mode = (m->plan & SI_PLAN_SELF_PREFETCH) ? 2 : (m->plan & SI_PLAN_FULL_RING) ? 1 : 0;
  qb.q1w = (m->plan & SI_PLAN_Q1_8WARPS) ? 8 : 16;
  const bool tp_fused = !(m->plan & SI_PLAN_TP_PREP_APART);
  // Each kernel may prefetch into L2 the weights of the kernel two launches
  // later: gate/up(l) -> qkv(l+1), down(l) -> Wo(l+1), attention(l) ->
  // gate/up(l), Wo(l) -> down(l).
  auto with_pf = [&](QmvBuffers q, const si_weight* w) {
    if (pre && w) q.pf = pf_of(w);
    return q;
  };
  {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = cfg_of(s, dim3((h + 255) / 256, B), dim3(256), 0, false, attr);
    SI_CUDA(cudaLaunchKernelEx(&cfg, k_embed, (const StepParams*)m->dparams, m->emb->qtype,
                               (const uint8_t*)m->emb->dev, m->emb->nblk, (int64_t)m->emb->rows, h, m->x));
  }
  for (int l = 0; l < L; l++) {
    const si_weight* qkv_next = l + 1 < L ? m->wqkv[l + 1] : nullptr;
    const si_weight* wo_next = l + 1 < L ? m->wo[l + 1] : nullptr;
    bool qkv_done = false, gu_done = false;  // matvecs that took their RmsNorm in
    if (tp && l > 0) {
      const PrepTp pt = tp_consumer(m, l - 1, 1);
      const int r = B == 1 && tp_fused ? launch_qmv_rms_tp(s, m->wqkv[l], m->x2, m->x, norm_ptr(m, l, SI_T_ATTN_NORM),
                                                          c.rms_eps, m->qkv, qb, pt, true)
                                       : -1;
      if (r > 0) return r;
      qkv_done = r == 0;
      if (!qkv_done)
        SI_TRY(launch_prep(s, m->x2, h, nullptr, norm_ptr(m, l, SI_T_ATTN_NORM), c.rms_eps, SI_PREP_RMSNORM_TP, h, B,
                           m->x, m->xprep, true, &pt));
    } else if (!tp && B == 1) {  // RmsNorm inside the matvec where the kernel allows
      SI_TRY(launch_qmv_rms(s, m->wqkv[l], m->x, norm_ptr(m, l, SI_T_ATTN_NORM), c.rms_eps, m->qkv, SI_EPI_STORE, qb,
                            m->xprep, true));
    } else {
      SI_TRY(launch_prep(s, m->x, h, nullptr, norm_ptr(m, l, SI_T_ATTN_NORM), c.rms_eps, SI_PREP_RMSNORM, h, B,
                         nullptr, m->xprep, true));
    }
    if ((tp || B > 1) && !qkv_done) SI_TRY(launch_qmv(s, m->wqkv[l], m->xprep, B, m->qkv, SI_EPI_STORE, qb, true));
    SI_TRY(enqueue_attention(m, l, m->qkv, nullptr, B, true, pre ? pf_of(m->wgu[l]) : L2Prefetch{}));
    if (tp) {
      SI_TRY(launch_qmv(s, m->wo[l], m->xprep, B, nullptr, SI_EPI_TP, with_pf(tp_producer(m, l, 0), m->wdown[l]),
                        true));
      const PrepTp pt = tp_consumer(m, l, 0);
      const int r = B == 1 && tp_fused ? launch_qmv_rms_tp(s, m->wgu[l], m->x, m->x2, norm_ptr(m, l, SI_T_FFN_NORM),
                                                          c.rms_eps, m->gu, with_pf(qb, qkv_next), pt, true)
                                       : -1;
      if (r > 0) return r;
      gu_done = r == 0;
      if (!gu_done)
        SI_TRY(launch_prep(s, m->x, h, nullptr, norm_ptr(m, l, SI_T_FFN_NORM), c.rms_eps, SI_PREP_RMSNORM_TP, h, B,
                           m->x2, m->xprep, true, &pt));
    } else {
      SI_TRY(launch_qmv(s, m->wo[l], m->xprep, B, m->x, SI_EPI_ADD, with_pf(qb, m->wdown[l]), true));
      if (B > 1)
        SI_TRY(launch_prep(s, m->x, h, nullptr, norm_ptr(m, l, SI_T_FFN_NORM), c.rms_eps, SI_PREP_RMSNORM, h, B,
                           nullptr, m->xprep, true));
    }
    if (!tp && B == 1)
      SI_TRY(launch_qmv_rms(s, m->wgu[l], m->x, norm_ptr(m, l, SI_T_FFN_NORM), c.rms_eps, m->gu, SI_EPI_STORE,
                            with_pf(qb, qkv_next), m->xprep, true));
    else if (!gu_done)
      SI_TRY(launch_qmv(s, m->wgu[l], m->xprep, B, m->gu, SI_EPI_STORE, with_pf(qb, qkv_next), true));
    if (B == 1 && (m->plan & SI_PLAN_SILU_IN_DOWN)) {  // SiLU(gate) * up inside the down-projection matvec
      if (tp)
        SI_TRY(launch_qmv_silu(s, m->wdown[l], m->gu, m->gu + inter, nullptr, SI_EPI_TP,
                               with_pf(tp_producer(m, l, 1), wo_next), m->xprep, true));
      else
        SI_TRY(launch_qmv_silu(s, m->wdown[l], m->gu, m->gu + inter, m->x, SI_EPI_ADD, with_pf(qb, wo_next),
                               m->xprep, true));
    } else {
      SI_TRY(launch_prep(s, m->gu, 2 * inter, m->gu + inter, nullptr, 0.f, SI_PREP_SILU_MUL, inter, B, nullptr,
                         m->xprep, true));
      if (tp)
        SI_TRY(launch_qmv(s, m->wdown[l], m->xprep, B, nullptr, SI_EPI_TP, with_pf(tp_producer(m, l, 1), wo_next),
                          true));
      else SI_TRY(launch_qmv(s, m->wdown[l], m->xprep, B, m->x, SI_EPI_ADD, with_pf(qb, wo_next), true));
    }
  }
  if (tp) {
    const PrepTp pt = tp_consumer(m, c.n_layers - 1, 1);
    SI_TRY(launch_prep(s, m->x2, h, nullptr, norm_ptr(m, -1, SI_T_FINAL_NORM), c.rms_eps, SI_PREP_RMSNORM_TP, h, B,
                       m->x, m->xprep, true, &pt));
  } else {
    SI_TRY(launch_prep(s, m->x, h, nullptr, norm_ptr(m, -1, SI_T_FINAL_NORM), c.rms_eps, SI_PREP_RMSNORM, h, B,
                       nullptr, m->xprep, true));
  }
  SI_TRY(launch_qmv(s, m->lm_head, m->xprep, B, m->logits, SI_EPI_STORE, qb, true));
  {
    ArgmaxTp at;
    if (tp) {
      at.peers = m->peers_dev;
      at.comm = m->comm;
      at.epoch = &m->dparams->epoch;
      at.err = m->c->dev_err;
      at.tp = m->tp;
      at.rank = m->rank;
    }
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = cfg_of(s, dim3(B), dim3(1024), 0, true, attr);
    SI_CUDA(cudaLaunchKernelEx(&cfg, k_argmax, (const float*)m->logits, (int64_t)c.vocab, m->argmax, at));
  }
  {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = cfg_of(s, dim3(1), dim3(SI_MAX_BATCH), 0, true, attr);
    SI_CUDA(cudaLaunchKernelEx(&cfg, k_advance, m->dparams, (const int*)m->argmax));
  }
  return SI_OK;
}

int get_graph(si_model* m, int B, cudaGraphExec_t* out) {
  auto it = m->graphs.find(B);
  if (it != m->graphs.end()) {
    *out = it->second;
    return SI_OK;
  }
  cudaStream_t s = m->c->stream;
  SI_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
  int st = enqueue_step(m, B);
  cudaGraph_t g = nullptr;
  cudaError_t e = cudaStreamEndCapture(s, &g);
  if (st != SI_OK) {
    if (g) cudaGraphDestroy(g);
    return st;
  }
  if (e != cudaSuccess) SI_FAIL(SI_ERR_CUDA, "decode-step capture failed: %s", cudaGetErrorString(e));
  size_t nn = 0;
  int kernels = 0;
  if (cudaGraphGetNodes(g, nullptr, &nn) == cudaSuccess && nn) {
    std::vector<cudaGraphNode_t> nodes(nn);
    if (cudaGraphGetNodes(g, nodes.data(), &nn) == cudaSuccess)
      for (auto nd : nodes) {
        cudaGraphNodeType ty;
        if (cudaGraphNodeGetType(nd, &ty) == cudaSuccess && ty == cudaGraphNodeTypeKernel) kernels++;
      }
  }
  m->graph_kernels[B] = kernels;
  cudaGraphExec_t ge = nullptr;
  e = cudaGraphInstantiate(&ge, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) SI_FAIL(SI_ERR_CUDA, "decode-step graph instantiation failed: %s", cudaGetErrorString(e));
  m->graphs[B] = ge;
  *out = ge;
  return SI_OK;
}

// Host-side cos/sin table with exactly the float arithmetic of
// RotaryEmbedding.ApplyToHead (RotaryEmbedding.cs:42-61): freq =
// 1 / powf(theta, i / headDim), angle = position * freq.
void fill_rope(std::vector<float>& t, int npos, int hd, float theta) {
  t.resize((size_t)npos * hd);
  for (int p = 0; p < npos; p++)
    for (int i = 0; i < hd; i += 2) {
      const float fi = (float)i / (float)hd;
      const float freq = 1.0f / powf(theta, fi);
      const float angle = (float)p * freq;
      t[((size_t)p * (hd / 2) + i / 2) * 2 + 0] = cosf(angle);
      t[((size_t)p * (hd / 2) + i / 2) * 2 + 1] = sinf(angle);
    }
}

}  // namespace

extern "C" {

SI_EXPORT int si_model_tensor_recipe(const si_model_config* c, int layer, int t, uint64_t* tag, int* qt,
                                     int* recipe, float* sigma, float* mean, int64_t* rows, int64_t* cols) {
  clear_error();
  SI_TRY(check_config(c));
  const int64_t hd = c->head_dim, qr = (int64_t)c->n_heads * hd, kr = (int64_t)c->n_kv_heads * hd;
  int64_t r = 0, k = 0;
  int q = c->weight_qtype, rc = SI_SYNTH_MODEL;
  float mu = 0.f, sg = 0.f;
  uint64_t tg;
  if (layer < 0) {
    tg = (uint64_t)(t - SI_T_EMB + 1);
    if (t == SI_T_EMB) { q = c->emb_qtype; r = c->vocab; k = c->hidden; }
    else if (t == SI_T_LM_HEAD) { q = c->lm_head_qtype; r = c->vocab; k = c->hidden; rc = SI_SYNTH_PLAIN; }
    else if (t == SI_T_FINAL_NORM) { q = SI_F32; r = 1; k = c->hidden; }
    else SI_FAIL(SI_ERR_INVALID, "unknown global tensor %d", t);
  } else {
    if (layer >= c->n_layers) SI_FAIL(SI_ERR_INVALID, "layer %d out of range", layer);
    tg = 1000ull * (uint64_t)(layer + 1) + (uint64_t)t;
    switch (t) {
      case SI_T_Q: r = qr; k = c->hidden; break;
      case SI_T_K: case SI_T_V: r = kr; k = c->hidden; break;
      case SI_T_O: r = c->hidden; k = qr; break;
      case SI_T_GATE: case SI_T_UP: r = c->intermediate; k = c->hidden; break;
      case SI_T_DOWN: r = c->hidden; k = c->intermediate; break;
      case SI_T_ATTN_NORM: case SI_T_FFN_NORM: q = SI_F32; r = 1; k = c->hidden; break;
      default: SI_FAIL(SI_ERR_INVALID, "unknown layer tensor %d", t);
    }
  }
  if (q == SI_F32) {
    mu = 1.0f;
    sg = 0.01f;
    rc = 0;
  } else if (t == SI_T_EMB) {
    sg = q == SI_Q4_K ? 1.0f / 23.3f : recipe_sigma(q, rc, 1);
  } else {
    sg = recipe_sigma(q, rc, k);
  }
  if (tag) *tag = tg;
  if (qt) *qt = q;
  if (recipe) *recipe = rc;
  if (sigma) *sigma = sg;
  if (mean) *mean = mu;
  if (rows) *rows = r;
  if (cols) *cols = k;
  return SI_OK;
}

SI_EXPORT uint64_t si_model_kv_tag(int layer, int seq, int is_value) {
  return 0x4B560000ull + ((uint64_t)layer * 64 + (uint64_t)seq) * 2 + (uint64_t)(is_value != 0);
}

SI_EXPORT int si_model_create_tp(si_ctx* ctx, const si_model_config* cfg, int tp, int rank, si_model** out) {
  clear_error();
  if (!ctx || !out) SI_FAIL(SI_ERR_INVALID, "si_model_create: NULL argument");
  *out = nullptr;
  SI_TRY(check_config(cfg));
  if (tp != 1 && tp != 2 && tp != 4 && tp != 8) SI_FAIL(SI_ERR_UNSUPPORTED, "tensor parallel size %d (1, 2, 4 or 8)", tp);
  if (rank < 0 || rank >= tp) SI_FAIL(SI_ERR_INVALID, "rank %d outside [0, %d)", rank, tp);
  {
    const int be = cfg->weight_qtype == SI_Q8_0 ? 32 : 256;
    if (cfg->n_kv_heads % tp || cfg->vocab % tp || (cfg->intermediate / tp) % be || (cfg->intermediate / tp) % 16 ||
        cfg->intermediate % tp || ((cfg->n_heads / tp) * cfg->head_dim) % be)
      SI_FAIL(SI_ERR_INVALID, "model shapes do not split over %d ranks on quant-block boundaries", tp);
  }
  SI_TRY(bind_device(ctx));
  si_model* m = new si_model();
  m->c = ctx;
  m->gcfg = *cfg;
  m->cfg = *cfg;
  m->tp = tp;
  m->rank = rank;
  m->plan = step_plan();
  m->cfg.n_heads /= tp;
  m->cfg.n_kv_heads /= tp;
  m->cfg.intermediate /= tp;
  m->cfg.vocab /= tp;
  const si_model_config& c = m->cfg;
  m->G = c.n_heads / c.n_kv_heads;
  m->qkv_rows = (c.n_heads + 2 * c.n_kv_heads) * c.head_dim;
  const int qd = c.n_heads * c.head_dim;
  m->Kmax = std::max(std::max(c.hidden, c.intermediate), qd);
  const int B = c.max_batch;
  int st = SI_OK;
  auto fail = [&](int code) {
    si_model_free(m);
    return code;
  };
  m->wqkv.assign(c.n_layers, nullptr);
  m->wo.assign(c.n_layers, nullptr);
  m->wgu.assign(c.n_layers, nullptr);
  m->wdown.assign(c.n_layers, nullptr);
  for (int l = 0; l < c.n_layers && st == SI_OK; l++) {
    st = make_weight(m, c.weight_qtype, m->qkv_rows, c.hidden, &m->wqkv[l]);
    if (st == SI_OK) st = make_weight(m, c.weight_qtype, c.hidden, qd, &m->wo[l]);
    if (st == SI_OK) st = make_weight(m, c.weight_qtype, 2 * (int64_t)c.intermediate, c.hidden, &m->wgu[l]);
    if (st == SI_OK) st = make_weight(m, c.weight_qtype, c.hidden, c.intermediate, &m->wdown[l]);
  }
  if (st == SI_OK) st = make_weight(m, c.emb_qtype, m->gcfg.vocab, c.hidden, &m->emb);
  if (st == SI_OK) st = make_weight(m, c.lm_head_qtype, c.vocab, c.hidden, &m->lm_head);
  if (st != SI_OK) return fail(st);
  const int64_t h = c.hidden;
  const size_t kv_elems = (size_t)c.n_layers * B * c.n_kv_heads * c.max_seq * c.head_dim;
  m->splits_max = std::min(511, std::max((2 * ctx->sm_count + c.n_kv_heads - 1) / c.n_kv_heads,
                                         (c.max_seq + 1023) / 1024 + 1));
  m->chunk_max = 1024;
  void* p;
#define ALLOC(field, bytes)                                      \
  do {                                                           \
    if ((st = dev_alloc(m, &p, (size_t)(bytes))) != SI_OK) return fail(st); \
    m->field = (decltype(m->field))p;                            \
  } while (0)
  ALLOC(norms, ((int64_t)c.n_layers * 2 + 1) * h * 4);
  ALLOC(kcache, kv_elems * 2);
  ALLOC(vcache, kv_elems * 2);
  ALLOC(rope, (size_t)c.max_seq * c.head_dim * 4);
  ALLOC(x, (size_t)B * h * 4);
  ALLOC(x2, (size_t)B * h * 4);
  if (tp > 1) {
    ALLOC(comm, SI_TP_SLOTS + (size_t)2 * tp * B * h * 8);
    ALLOC(peers_dev, SI_TP_MAX * sizeof(uint8_t*));
  }
  ALLOC(qkv, (size_t)B * m->qkv_rows * 4);
  ALLOC(gu, (size_t)B * 2 * c.intermediate * 4);
  ALLOC(logits, (size_t)B * c.vocab * 4);
  ALLOC(argmax, (size_t)SI_MAX_BATCH * 4);
  ALLOC(xprep, xprep_bytes(m->Kmax, B));
  ALLOC(part_o, (size_t)B * c.n_heads * m->splits_max * c.head_dim * 4);
  ALLOC(part_ml, (size_t)B * c.n_heads * m->splits_max * 2 * 4);
  ALLOC(merge_cnt, (size_t)B * c.n_kv_heads * 4);
  ALLOC(dparams, sizeof(StepParams));
#undef ALLOC
  cudaError_t e = cudaMemset(m->kcache, 0, kv_elems * 2);
  if (e == cudaSuccess && m->comm) e = cudaMemset(m->comm, 0, SI_TP_SLOTS + (size_t)2 * tp * B * h * 8);
  if (e == cudaSuccess) e = cudaMemset(m->vcache, 0, kv_elems * 2);
  if (e == cudaSuccess) e = cudaMemset(m->merge_cnt, 0, (size_t)B * c.n_kv_heads * 4);
  if (e == cudaSuccess) e = cudaMallocHost(&m->hparams, sizeof(StepParams));
  if (e == cudaSuccess) e = cudaMallocHost(&m->hargmax, sizeof(int) * SI_MAX_BATCH);
  if (e != cudaSuccess) {
    si::set_error("model set-up failed: %s", cudaGetErrorString(e));
    return fail(SI_ERR_CUDA);
  }
  std::vector<float> rope;
  fill_rope(rope, c.max_seq, c.head_dim, c.rope_theta);
  e = cudaMemcpy(m->rope, rope.data(), rope.size() * 4, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    si::set_error("rope table upload failed: %s", cudaGetErrorString(e));
    return fail(SI_ERR_CUDA);
  }
  for (si_weight* w : {m->wqkv[0], m->wo[0], m->wgu[0], m->wdown[0], m->lm_head})
    if ((st = ensure_qmv_scratch(ctx, w)) != SI_OK) return fail(st);
  *out = m;
  return SI_OK;
}

SI_EXPORT int si_model_get_config(const si_model* m, si_model_config* out) {
  clear_error();
  if (!m || !out) SI_FAIL(SI_ERR_INVALID, "si_model_get_config: NULL argument");
  *out = m->gcfg;
  return SI_OK;
}

SI_EXPORT int si_model_create(si_ctx* ctx, const si_model_config* cfg, si_model** out) {
  return si_model_create_tp(ctx, cfg, 1, 0, out);
}

SI_EXPORT int si_tp_slice(const si_model_config* cfg, int tp, int rank, int tensor, int64_t* grow0, int64_t* rows,
                          int64_t* gb0, int64_t* nblk, int64_t* gnblk) {
  clear_error();
  if (!cfg || !grow0 || !rows || !gb0 || !nblk || !gnblk) SI_FAIL(SI_ERR_INVALID, "si_tp_slice: NULL argument");
  if (tp < 1 || rank < 0 || rank >= tp) SI_FAIL(SI_ERR_INVALID, "si_tp_slice: rank %d of %d", rank, tp);
  return tp_slice(*cfg, tp, rank, tensor, grow0, rows, gb0, nblk, gnblk);
}

SI_EXPORT int si_model_tp_handle(si_model* m, void* handle_out, int len) {
  clear_error();
  if (!m || !handle_out || len < (int)sizeof(cudaIpcMemHandle_t))
    SI_FAIL(SI_ERR_INVALID, "si_model_tp_handle: need %d bytes", (int)sizeof(cudaIpcMemHandle_t));
  if (m->tp == 1) SI_FAIL(SI_ERR_INVALID, "si_model_tp_handle: model is not tensor parallel");
  SI_TRY(bind_device(m->c));
  cudaIpcMemHandle_t h;
  SI_CUDA(cudaIpcGetMemHandle(&h, m->comm));
  memcpy(handle_out, &h, sizeof(h));
  return SI_OK;
}

SI_EXPORT int si_model_tp_connect(si_model* m, const void* handles, int len) {
  clear_error();
  if (!m || !handles) SI_FAIL(SI_ERR_INVALID, "si_model_tp_connect: NULL argument");
  const int hs = (int)sizeof(cudaIpcMemHandle_t);
  if (m->tp == 1 || len != m->tp * hs) SI_FAIL(SI_ERR_INVALID, "si_model_tp_connect: need %d handles", m->tp);
  if (m->connected) SI_FAIL(SI_ERR_INVALID, "si_model_tp_connect: already connected");
  SI_TRY(bind_device(m->c));
  for (int r = 0; r < m->tp; r++) {
    if (r == m->rank) {
      m->peer_base[r] = m->comm;
      continue;
    }
    cudaIpcMemHandle_t h;
    memcpy(&h, (const uint8_t*)handles + r * hs, hs);
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int q = 0; q < r; q++)
        if (q != m->rank && m->peer_base[q]) cudaIpcCloseMemHandle(m->peer_base[q]);
      SI_FAIL(SI_ERR_CUDA, "opening rank %d's buffer failed: %s", r, cudaGetErrorString(e));
    }
    m->peer_base[r] = (uint8_t*)p;
  }
  m->ipc = true;
  SI_CUDA(cudaMemcpy(m->peers_dev, m->peer_base, SI_TP_MAX * sizeof(uint8_t*), cudaMemcpyHostToDevice));
  m->connected = true;
  return SI_OK;
}

SI_EXPORT int si_model_tp_connect_local(si_model* m, si_model* const* ranks, int n) {
  clear_error();
  if (!m || !ranks) SI_FAIL(SI_ERR_INVALID, "si_model_tp_connect_local: NULL argument");
  if (m->tp == 1 || n != m->tp) SI_FAIL(SI_ERR_INVALID, "si_model_tp_connect_local: need %d ranks", m->tp);
  if (m->connected) SI_FAIL(SI_ERR_INVALID, "si_model_tp_connect_local: already connected");
  for (int r = 0; r < n; r++) {
    const si_model* o = ranks[r];
    if (!o || o->tp != m->tp || o->rank != r || memcmp(&o->gcfg, &m->gcfg, sizeof(si_model_config)) != 0)
      SI_FAIL(SI_ERR_INVALID, "si_model_tp_connect_local: entry %d is not rank %d of the same model", r, r);
  }
  SI_TRY(bind_device(m->c));
  for (int r = 0; r < n; r++) {
    const int pd = ranks[r]->c->device;
    if (pd != m->c->device) {
      int can = 0;
      SI_CUDA(cudaDeviceCanAccessPeer(&can, m->c->device, pd));
      if (!can) SI_FAIL(SI_ERR_UNSUPPORTED, "device %d cannot access device %d's memory", m->c->device, pd);
      const cudaError_t e = cudaDeviceEnablePeerAccess(pd, 0);
      if (e == cudaErrorPeerAccessAlreadyEnabled) cudaGetLastError();
      else if (e != cudaSuccess) SI_FAIL(SI_ERR_CUDA, "enabling access to device %d failed: %s", pd, cudaGetErrorString(e));
    }
    m->peer_base[r] = ranks[r]->comm;
  }
  m->ipc = false;
  SI_CUDA(cudaMemcpy(m->peers_dev, m->peer_base, SI_TP_MAX * sizeof(uint8_t*), cudaMemcpyHostToDevice));
  m->connected = true;
  return SI_OK;
}

SI_EXPORT int si_model_free(si_model* m) {
  clear_error();
  if (!m) return SI_OK;
  cudaSetDevice(m->c->device);
  cudaStreamSynchronize(m->c->stream);
  for (auto& kv : m->graphs) cudaGraphExecDestroy(kv.second);
  if (m->connected && m->ipc)
    for (int r = 0; r < m->tp; r++)
      if (r != m->rank && m->peer_base[r]) cudaIpcCloseMemHandle(m->peer_base[r]);
  for (auto* v : {&m->wqkv, &m->wo, &m->wgu, &m->wdown})
    for (si_weight* w : *v) si_weight_free(w);
  si_weight_free(m->emb);
  si_weight_free(m->lm_head);
  for (void* p : m->allocs) cudaFree(p);
  for (si_devbuf* b : {&m->pf_tok, &m->pf_x, &m->pf_xh, &m->pf_rs, &m->pf_qkv, &m->pf_gu, &m->pf_q, &m->pf_k, &m->pf_v,
                       &m->pf_o})
    if (b->ptr) cudaFree(b->ptr);
  if (m->hparams) cudaFreeHost(m->hparams);
  if (m->hargmax) cudaFreeHost(m->hargmax);
  if (m->hist) cudaFree(m->hist);
  delete m;
  return SI_OK;
}

SI_EXPORT int si_model_set_tensor(si_model* m, int layer, int t, const void* host) {
  clear_error();
  if (!m || !host) SI_FAIL(SI_ERR_INVALID, "si_model_set_tensor: NULL argument");
  si_ctx* c = m->c;
  SI_TRY(bind_device(c));
  if (t == SI_T_ATTN_NORM || t == SI_T_FFN_NORM || t == SI_T_FINAL_NORM) {
    if ((layer < 0) != (t == SI_T_FINAL_NORM)) SI_FAIL(SI_ERR_INVALID, "norm tensor %d with layer %d", t, layer);
    if (layer >= m->cfg.n_layers) SI_FAIL(SI_ERR_INVALID, "layer %d out of range", layer);
    SI_CUDA(cudaMemcpy(norm_ptr(m, layer, t), host, (size_t)m->cfg.hidden * 4, cudaMemcpyHostToDevice));
    return SI_OK;
  }
  Slot sl;
  SI_TRY(tensor_slot(m, layer, t, &sl));
  si_weight* w = sl.w;
  const int64_t bb = gguf_block_bytes(w->qtype);
  const int64_t rb = w->nblk * bb;                                // local bytes per row
  const uint8_t* src = (const uint8_t*)host + sl.grow0 * sl.gnblk * bb;
  const int64_t cr = std::max<int64_t>(16, ((64ll << 20) / rb) / 16 * 16);
  const int64_t rows = sl.rows;
  SI_TRY(ensure(c->stage[0], (size_t)(std::min(cr, rows) * rb)));
  std::vector<uint8_t> gather;
  for (int64_t r = 0; r < rows; r += cr) {
    const int64_t nr = std::min(cr, rows - r);
    const uint8_t* chunk = src + r * sl.gnblk * bb;
    if (sl.gnblk != w->nblk) {  // a slice of every row: gather it on the host
      gather.resize((size_t)(nr * rb));
      for (int64_t i = 0; i < nr; i++)
        memcpy(gather.data() + i * rb, chunk + (i * sl.gnblk + sl.gb0) * bb, (size_t)rb);
      chunk = gather.data();
    }
    SI_CUDA(cudaMemcpyAsync(c->stage[0].ptr, chunk, (size_t)(nr * rb), cudaMemcpyHostToDevice, c->stream));
    SI_TRY(launch_repack(c, w->qtype, (const uint8_t*)c->stage[0].ptr, sl.row0 + rows, w->cols, sl.row0 + r, nr,
                         w->dev));
    SI_CUDA(cudaStreamSynchronize(c->stream));
  }
  return SI_OK;
}

SI_EXPORT int si_model_synth(si_model* m, uint64_t seed) {
  clear_error();
  if (!m) SI_FAIL(SI_ERR_INVALID, "si_model_synth: NULL model");
  si_ctx* c = m->c;
  SI_TRY(bind_device(c));
  const si_model_config& cfg = m->gcfg;  // recipes (tags, scales) are those of the whole tensors
  std::vector<std::pair<int, int>> items;
  for (int l = 0; l < cfg.n_layers; l++)
    for (int t = SI_T_Q; t <= SI_T_FFN_NORM; t++) items.push_back({l, t});
  for (int t : {SI_T_EMB, SI_T_LM_HEAD, SI_T_FINAL_NORM}) items.push_back({-1, t});
  for (auto& it : items) {
    const int layer = it.first, t = it.second;
    uint64_t tag;
    int qt, rc;
    float sg, mu;
    int64_t rows, cols;
    SI_TRY(si_model_tensor_recipe(&cfg, layer, t, &tag, &qt, &rc, &sg, &mu, &rows, &cols));
    if (qt == SI_F32) {
      const int64_t n = cols;
      k_f32_synth<<<(unsigned)((n + 255) / 256), 256, 0, c->stream>>>(norm_ptr(m, layer, t), si_key(seed, tag), n,
                                                                      mu, sg);
      SI_CUDA(cudaGetLastError());
      continue;
    }
    Slot sl;
    SI_TRY(tensor_slot(m, layer, t, &sl));
    si_weight* w = sl.w;
    const int64_t rl = sl.rows;
    const int64_t rb = w->nblk * gguf_block_bytes(qt);
    const int64_t cr = std::max<int64_t>(16, ((64ll << 20) / rb) / 16 * 16);
    SI_TRY(ensure(c->stage[0], (size_t)(std::min(cr, rl) * rb)));
    for (int64_t r = 0; r < rl; r += cr) {
      const int64_t nr = std::min(cr, rl - r);
      // global blocks (grow0 + r + i) * gnblk + gb0 + j, j < nblk, in local row-major order
      SI_TRY(launch_synth_blocks_2d(c, qt, seed, tag, rc, sg, sl.grow0 + r, nr, sl.gnblk, sl.gb0, w->nblk,
                                    (uint8_t*)c->stage[0].ptr));
      SI_TRY(launch_repack(c, qt, (const uint8_t*)c->stage[0].ptr, sl.row0 + rl, w->cols, sl.row0 + r, nr, w->dev));
      SI_CUDA(cudaStreamSynchronize(c->stream));
    }
  }
  SI_CUDA(cudaStreamSynchronize(c->stream));
  return SI_OK;
}

SI_EXPORT int si_model_kv_synth(si_model* m, int len, uint64_t seed) {
  clear_error();
  if (!m) SI_FAIL(SI_ERR_INVALID, "si_model_kv_synth: NULL model");
  const si_model_config& c = m->cfg;
  if (len < 0 || len > c.max_seq) SI_FAIL(SI_ERR_INVALID, "kv length %d outside [0, %d]", len, c.max_seq);
  SI_TRY(bind_device(m->c));
  const int64_t per = (int64_t)c.n_kv_heads * c.max_seq * c.head_dim;
  const int64_t n = (int64_t)len * c.n_kv_heads * c.head_dim;
  if (n == 0) return SI_OK;
  for (int l = 0; l < c.n_layers; l++)
    for (int b = 0; b < c.max_batch; b++) {
      const int64_t off = ((int64_t)l * c.max_batch + b) * per;
      for (int v = 0; v < 2; v++) {
        __half* base = (v ? m->vcache : m->kcache) + off;
        k_kv_synth<<<(unsigned)((n + 255) / 256), 256, 0, m->c->stream>>>(
            base, si_key(seed, si_model_kv_tag(l, b, v)), len, c.n_kv_heads, c.max_seq, m->gcfg.n_kv_heads,
            m->rank * c.n_kv_heads);
      }
    }
  SI_CUDA(cudaGetLastError());
  SI_CUDA(cudaStreamSynchronize(m->c->stream));
  return SI_OK;
}

SI_EXPORT int si_model_kv_write(si_model* m, int layer, int seq, int pos0, int n, const uint16_t* k,
                                const uint16_t* v) {
  clear_error();
  if (!m || !k || !v) SI_FAIL(SI_ERR_INVALID, "si_model_kv_write: NULL argument");
  const si_model_config& c = m->cfg;
  if (layer < 0 || layer >= c.n_layers || seq < 0 || seq >= c.max_batch || pos0 < 0 || n < 0 ||
      pos0 + n > c.max_seq)
    SI_FAIL(SI_ERR_INVALID, "si_model_kv_write: range outside the cache");
  si_ctx* ctx = m->c;
  SI_TRY(bind_device(ctx));
  const size_t bytes = (size_t)n * m->gcfg.n_kv_heads * c.head_dim * 2;  // all kv heads, [n][heads][dim]
  if (!bytes) return SI_OK;
  SI_TRY(ensure(ctx->stage[3], bytes));
  const int64_t per = (int64_t)c.n_kv_heads * c.max_seq * c.head_dim;
  const int64_t off = ((int64_t)layer * c.max_batch + seq) * per;
  const int64_t cnt = (int64_t)n * c.n_kv_heads * c.head_dim;
  for (int which = 0; which < 2; which++) {
    SI_CUDA(cudaMemcpyAsync(ctx->stage[3].ptr, which ? v : k, bytes, cudaMemcpyHostToDevice, ctx->stream));
    k_kv_scatter<<<(unsigned)((cnt + 255) / 256), 256, 0, ctx->stream>>>(
        (which ? m->vcache : m->kcache) + off, (const uint16_t*)ctx->stage[3].ptr, pos0, n, c.n_kv_heads, c.max_seq,
        m->gcfg.n_kv_heads, m->rank * c.n_kv_heads);
    SI_CUDA(cudaGetLastError());
    SI_CUDA(cudaStreamSynchronize(ctx->stream));
  }
  return SI_OK;
}

SI_EXPORT int si_decode_step(si_model* m, const int* tokens, int batch, int pos, int* argmax_out,
                             float* logits_out) {
  clear_error();
  if (!m || !tokens || !argmax_out) SI_FAIL(SI_ERR_INVALID, "si_decode_step: NULL argument");
  const si_model_config& c = m->cfg;
  if (batch < 1 || batch > c.max_batch) SI_FAIL(SI_ERR_INVALID, "batch %d outside 1..%d", batch, c.max_batch);
  if (pos < 0 || pos >= c.max_seq)
    SI_FAIL(SI_ERR_INVALID, "position %d exceeds max sequence length %d", pos, c.max_seq);  // KVCache.cs:48-49
  for (int b = 0; b < batch; b++)
    if (tokens[b] < 0 || tokens[b] >= m->gcfg.vocab)
      SI_FAIL(SI_ERR_INVALID, "token id %d outside the vocabulary", tokens[b]);
  if (m->tp > 1 && !m->connected) SI_FAIL(SI_ERR_INVALID, "tensor-parallel model not connected to its peers");
  SI_TRY(bind_device(m->c));
  cudaGraphExec_t ge;
  SI_TRY(get_graph(m, batch, &ge));
  m->hparams->epoch = m->epoch++;
  m->hparams->pos = pos;
  m->hparams->batch = batch;
  for (int b = 0; b < batch; b++) m->hparams->tokens[b] = tokens[b];
  m->hparams->step = 0;
  m->hparams->hist_cap = 0;
  m->hparams->hist = nullptr;
  cudaStream_t s = m->c->stream;
  SI_CUDA(cudaMemcpyAsync(m->dparams, m->hparams, sizeof(StepParams), cudaMemcpyHostToDevice, s));
  SI_CUDA(cudaGraphLaunch(ge, s));
  SI_CUDA(cudaMemcpyAsync(m->hargmax, m->argmax, sizeof(int) * batch, cudaMemcpyDeviceToHost, s));
  if (logits_out)
    SI_CUDA(cudaMemcpyAsync(logits_out, m->logits, (size_t)batch * c.vocab * 4, cudaMemcpyDeviceToHost, s));
  SI_CUDA(cudaStreamSynchronize(s));
  SI_TRY(check_device_errors(m->c));
  for (int b = 0; b < batch; b++) argmax_out[b] = m->hargmax[b];
  return SI_OK;
}

SI_EXPORT int si_decode_generate(si_model* m, const int* tokens, int batch, int pos0, int nsteps,
                                 int* out_tokens) {
  clear_error();
  if (!m || !tokens || !out_tokens) SI_FAIL(SI_ERR_INVALID, "si_decode_generate: NULL argument");
  const si_model_config& c = m->cfg;
  if (batch < 1 || batch > c.max_batch) SI_FAIL(SI_ERR_INVALID, "batch %d outside 1..%d", batch, c.max_batch);
  if (nsteps < 0 || pos0 < 0 || (int64_t)pos0 + nsteps > c.max_seq)
    SI_FAIL(SI_ERR_INVALID, "positions %d..%d exceed max sequence length %d", pos0, pos0 + nsteps, c.max_seq);
  for (int b = 0; b < batch; b++)
    if (tokens[b] < 0 || tokens[b] >= m->gcfg.vocab)
      SI_FAIL(SI_ERR_INVALID, "token id %d outside the vocabulary", tokens[b]);
  if (m->tp > 1 && !m->connected) SI_FAIL(SI_ERR_INVALID, "tensor-parallel model not connected to its peers");
  if (nsteps == 0) return SI_OK;
  SI_TRY(bind_device(m->c));
  cudaGraphExec_t ge;
  SI_TRY(get_graph(m, batch, &ge));
  const int64_t need = (int64_t)nsteps * batch;
  if (need > m->hist_cap) {
    if (m->hist) cudaFree(m->hist);
    m->hist = nullptr;
    m->hist_cap = 0;
    SI_CUDA(cudaMalloc(&m->hist, (size_t)need * 4));
    m->hist_cap = need;
  }
  m->hparams->epoch = m->epoch;
  m->epoch += (unsigned)nsteps;
  m->hparams->pos = pos0;
  m->hparams->batch = batch;
  for (int b = 0; b < batch; b++) m->hparams->tokens[b] = tokens[b];
  m->hparams->step = 0;
  m->hparams->hist_cap = nsteps;
  m->hparams->hist = m->hist;
  cudaStream_t s = m->c->stream;
  SI_CUDA(cudaMemcpyAsync(m->dparams, m->hparams, sizeof(StepParams), cudaMemcpyHostToDevice, s));
  for (int i = 0; i < nsteps; i++) SI_CUDA(cudaGraphLaunch(ge, s));
  SI_CUDA(cudaMemcpyAsync(out_tokens, m->hist, (size_t)need * 4, cudaMemcpyDeviceToHost, s));
  SI_CUDA(cudaStreamSynchronize(s));
  return check_device_errors(m->c);
}

SI_EXPORT int si_decode_step_kernels(si_model* m, int batch, int* kernels) {
  clear_error();
  if (!m || !kernels) SI_FAIL(SI_ERR_INVALID, "si_decode_step_kernels: NULL argument");
  if (batch < 1 || batch > m->cfg.max_batch) SI_FAIL(SI_ERR_INVALID, "si_decode_step_kernels: batch %d", batch);
  SI_TRY(bind_device(m->c));
  cudaGraphExec_t ge;
  SI_TRY(get_graph(m, batch, &ge));
  *kernels = m->graph_kernels[batch];
  return SI_OK;
}

SI_EXPORT int si_model_prefill(si_model* m, int seq, const int* tokens, int n, int pos0, int* argmax_out,
                               float* logits_out) {
  clear_error();
  if (!m || !tokens) SI_FAIL(SI_ERR_INVALID, "si_model_prefill: NULL argument");
  const si_model_config& c = m->cfg;
  if (m->tp > 1) SI_FAIL(SI_ERR_UNSUPPORTED, "si_model_prefill: tensor-parallel models prefill through si_decode_step");
  if (seq < 0 || seq >= c.max_batch) SI_FAIL(SI_ERR_INVALID, "si_model_prefill: sequence %d outside 0..%d", seq,
                                                c.max_batch - 1);
  if (n < 1 || pos0 < 0 || (int64_t)pos0 + n > c.max_seq)
    SI_FAIL(SI_ERR_INVALID, "si_model_prefill: positions %d..%d exceed max sequence length %d", pos0, pos0 + n,
            c.max_seq);  // KVCache.cs:48-49
  for (int i = 0; i < n; i++)
    if (tokens[i] < 0 || tokens[i] >= c.vocab) SI_FAIL(SI_ERR_INVALID, "token id %d outside the vocabulary", tokens[i]);
  si_ctx* ctx = m->c;
  SI_TRY(bind_device(ctx));
  cudaStream_t s = ctx->stream;
  const int h = c.hidden, inter = c.intermediate, nh = c.n_heads, nkv = c.n_kv_heads, L = pos0 + n;
  const int kmax = std::max(std::max(h, inter), nh * c.head_dim);
  SI_TRY(ensure(m->pf_tok, (size_t)n * 4));
  SI_TRY(ensure(m->pf_x, (size_t)n * h * 4));
  SI_TRY(ensure(m->pf_xh, (size_t)n * kmax * 2));
  SI_TRY(ensure(m->pf_rs, (size_t)n * 4));
  SI_TRY(ensure(m->pf_qkv, (size_t)n * m->qkv_rows * 4));
  SI_TRY(ensure(m->pf_gu, (size_t)n * 2 * inter * 4));
  SI_TRY(ensure(m->pf_q, (size_t)nh * n * c.head_dim * 2));
  SI_TRY(ensure(m->pf_k, (size_t)nkv * L * c.head_dim * 2));
  SI_TRY(ensure(m->pf_v, (size_t)nkv * L * c.head_dim * 2));
  SI_TRY(ensure(m->pf_o, (size_t)nh * n * c.head_dim * 4));
  float* x = (float*)m->pf_x.ptr;
  __half* xh = (__half*)m->pf_xh.ptr;
  float* rs = (float*)m->pf_rs.ptr;
  float* qkv = (float*)m->pf_qkv.ptr;
  float* gu = (float*)m->pf_gu.ptr;
  __half* qh = (__half*)m->pf_q.ptr;
  __half* kd = (__half*)m->pf_k.ptr;
  __half* vd = (__half*)m->pf_v.ptr;
  float* o = (float*)m->pf_o.ptr;
  SI_CUDA(cudaMemcpyAsync(m->pf_tok.ptr, tokens, (size_t)n * 4, cudaMemcpyHostToDevice, s));
  SI_TRY(launch_embed_rows(s, (const int*)m->pf_tok.ptr, n, m->emb, h, x));
  const int64_t per = (int64_t)nkv * c.max_seq * c.head_dim;
  const float scale = 1.0f / sqrtf((float)c.head_dim);  // Transformer.cs:101
  for (int l = 0; l < c.n_layers; l++) {
    __half* kc = m->kcache + ((int64_t)l * c.max_batch + seq) * per;
    __half* vc = m->vcache + ((int64_t)l * c.max_batch + seq) * per;
    SI_TRY(launch_rms_rows(s, x, n, h, norm_ptr(m, l, SI_T_ATTN_NORM), c.rms_eps, xh, rs));
    SI_TRY(launch_qgemm_f16in(ctx, m->wqkv[l], xh, rs, qkv, n, 0));
    SI_TRY(launch_rope_store(s, qkv, m->qkv_rows, m->rope, pos0, n, nh, nkv, kc, vc, c.max_seq, qh));
    SI_TRY(launch_cache_dense(s, kc, c.max_seq, L, nkv, kd));
    SI_TRY(launch_cache_dense(s, vc, c.max_seq, L, nkv, vd));
    SI_TRY(launch_attn_prefill(ctx, (const uint16_t*)qh, (const uint16_t*)kd, (const uint16_t*)vd, o, 1, nh, nkv, n, L,
                               scale, 1, pos0, true));
    SI_TRY(launch_heads_rows(s, o, n, nh, xh, rs));
    SI_TRY(launch_qgemm_f16in(ctx, m->wo[l], xh, rs, x, n, 1));
    SI_TRY(launch_rms_rows(s, x, n, h, norm_ptr(m, l, SI_T_FFN_NORM), c.rms_eps, xh, rs));
    SI_TRY(launch_qgemm_f16in(ctx, m->wgu[l], xh, rs, gu, n, 0));
    SI_TRY(launch_silu_rows(s, gu, n, inter, xh, rs));
    SI_TRY(launch_qgemm_f16in(ctx, m->wdown[l], xh, rs, x, n, 1));
  }
  // the last prompt token's logits: final RmsNorm, lm_head, greedy ArgMax (Transformer.cs:158-159)
  SI_TRY(launch_prep(s, x + (int64_t)(n - 1) * h, h, nullptr, norm_ptr(m, -1, SI_T_FINAL_NORM), c.rms_eps,
                     SI_PREP_RMSNORM, h, 1, nullptr, m->xprep, false));
  SI_TRY(launch_qmv(s, m->lm_head, m->xprep, 1, m->logits, SI_EPI_STORE, ctx->qmv(), false));
  k_argmax<<<1, 1024, 0, s>>>((const float*)m->logits, (int64_t)c.vocab, m->argmax, ArgmaxTp{});
  SI_CUDA(cudaGetLastError());
  SI_CUDA(cudaMemcpyAsync(m->hargmax, m->argmax, sizeof(int), cudaMemcpyDeviceToHost, s));
  if (logits_out) SI_CUDA(cudaMemcpyAsync(logits_out, m->logits, (size_t)c.vocab * 4, cudaMemcpyDeviceToHost, s));
  SI_CUDA(cudaStreamSynchronize(s));
  SI_TRY(check_device_errors(ctx));
  if (argmax_out) *argmax_out = m->hargmax[0];
  return SI_OK;
}

SI_EXPORT int si_model_kv_read(si_model* m, int layer, int seq, int pos0, int n, uint16_t* k, uint16_t* v) {
  clear_error();
  if (!m || !k || !v) SI_FAIL(SI_ERR_INVALID, "si_model_kv_read: NULL argument");
  const si_model_config& c = m->cfg;
  if (layer < 0 || layer >= c.n_layers || seq < 0 || seq >= c.max_batch || pos0 < 0 || n < 0 || pos0 + n > c.max_seq)
    SI_FAIL(SI_ERR_INVALID, "si_model_kv_read: range outside the cache");
  if (n == 0) return SI_OK;
  si_ctx* ctx = m->c;
  SI_TRY(bind_device(ctx));
  const int64_t per = (int64_t)c.n_kv_heads * c.max_seq * c.head_dim;
  const int64_t off = ((int64_t)layer * c.max_batch + seq) * per;
  const size_t bytes = (size_t)c.n_kv_heads * (pos0 + n) * c.head_dim * 2;
  SI_TRY(ensure(ctx->stage[3], bytes));
  std::vector<uint16_t> dense((size_t)c.n_kv_heads * (pos0 + n) * c.head_dim);
  for (int which = 0; which < 2; which++) {
    SI_TRY(launch_cache_dense(ctx->stream, (which ? m->vcache : m->kcache) + off, c.max_seq, pos0 + n, c.n_kv_heads,
                              (__half*)ctx->stage[3].ptr));
    SI_CUDA(cudaMemcpyAsync(dense.data(), ctx->stage[3].ptr, bytes, cudaMemcpyDeviceToHost, ctx->stream));
    SI_CUDA(cudaStreamSynchronize(ctx->stream));
    uint16_t* out = which ? v : k;  // [n][kv head][dim], KVCache.cs:60-71
    for (int t = 0; t < n; t++)
      for (int kvh = 0; kvh < c.n_kv_heads; kvh++)
        memcpy(out + ((size_t)t * c.n_kv_heads + kvh) * c.head_dim,
               dense.data() + ((size_t)kvh * (pos0 + n) + pos0 + t) * c.head_dim, (size_t)c.head_dim * 2);
  }
  return SI_OK;
}

SI_EXPORT int si_model_kv_export(si_model* m, int seq, int length, void* out, size_t out_bytes) {
  clear_error();
  if (!m || !out) SI_FAIL(SI_ERR_INVALID, "si_model_kv_export: NULL argument");
  const si_model_config& c = m->cfg;
  if (m->tp > 1) SI_FAIL(SI_ERR_UNSUPPORTED, "si_model_kv_export: export each rank's model on a single-device copy");
  const size_t stride = (size_t)c.n_kv_heads * c.head_dim;
  const size_t need = (size_t)c.n_layers * 2 * length * stride * 4;
  if (length < 0 || length > c.max_seq || out_bytes < need)
    SI_FAIL(SI_ERR_INVALID, "si_model_kv_export: %d positions need %zu bytes", length, need);
  std::vector<uint16_t> k((size_t)length * stride), v((size_t)length * stride);
  float* dst = (float*)out;
  for (int l = 0; l < c.n_layers; l++) {  // KVCache.WriteRawData: per layer K then V, f32 [pos][kv head][dim]
    SI_TRY(si_model_kv_read(m, l, seq, 0, length, k.data(), v.data()));
    for (size_t i = 0; i < k.size(); i++) dst[i] = __half2float(__ushort_as_half(k[i]));
    dst += k.size();
    for (size_t i = 0; i < v.size(); i++) dst[i] = __half2float(__ushort_as_half(v[i]));
    dst += v.size();
  }
  return SI_OK;
}

SI_EXPORT int si_model_kv_import(si_model* m, int seq, int length, const void* in, size_t in_bytes) {
  clear_error();
  if (!m || !in) SI_FAIL(SI_ERR_INVALID, "si_model_kv_import: NULL argument");
  const si_model_config& c = m->cfg;
  if (m->tp > 1) SI_FAIL(SI_ERR_UNSUPPORTED, "si_model_kv_import: import on a single-device model");
  const size_t stride = (size_t)c.n_kv_heads * c.head_dim;
  const size_t need = (size_t)c.n_layers * 2 * length * stride * 4;
  if (length < 0 || length > c.max_seq || in_bytes < need)
    SI_FAIL(SI_ERR_INVALID, "si_model_kv_import: %d positions need %zu bytes", length, need);
  std::vector<uint16_t> k((size_t)length * stride), v((size_t)length * stride);
  const float* src = (const float*)in;
  for (int l = 0; l < c.n_layers; l++) {  // KVCache.ReadRawData, values rounded to the f16 cache
    for (size_t i = 0; i < k.size(); i++) k[i] = __half_as_ushort(__float2half_rn(src[i]));
    src += k.size();
    for (size_t i = 0; i < v.size(); i++) v[i] = __half_as_ushort(__float2half_rn(src[i]));
    src += v.size();
    SI_TRY(si_model_kv_write(m, l, seq, 0, length, k.data(), v.data()));
  }
  return SI_OK;
}

SI_EXPORT int si_model_attention(si_model* m, int layer, const float* qkv, float* out, int batch, int pos) {
  clear_error();
  if (!m || !qkv || !out) SI_FAIL(SI_ERR_INVALID, "si_model_attention: NULL argument");
  const si_model_config& c = m->cfg;
  if (layer < 0 || layer >= c.n_layers || batch < 1 || batch > c.max_batch || pos < 0 || pos >= c.max_seq)
    SI_FAIL(SI_ERR_INVALID, "si_model_attention: bad layer/batch/position");
  SI_TRY(bind_device(m->c));
  m->hparams->pos = pos;
  m->hparams->batch = batch;
  SI_CUDA(cudaMemcpyAsync(m->dparams, m->hparams, sizeof(StepParams), cudaMemcpyHostToDevice, m->c->stream));
  SI_TRY(enqueue_attention(m, layer, qkv, out, batch, false));
  SI_CUDA(cudaStreamSynchronize(m->c->stream));
  return check_device_errors(m->c);
}

}  // extern "C"
