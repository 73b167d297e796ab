/*
 * sharpinfer_b200 -- C ABI of the B200 (sm_100a) K-quant inference library.
 *
 * This is the native side of SharpInfer's compute-backend boundary.  The
 * reference binds a library named `sharpinfer_cuda` from C# with P/Invoke
 * (src/SharpInfer.Gpu/CudaBackend.cs:139-164,
 * src/SharpInfer.Core/Layers/FlashAttention.cs:378-385,
 * src/SharpInfer.Core/Tensors/HardwareBackends.cs:436-443) and calls it
 * through IComputeBackend (src/SharpInfer.Core/Tensors/TensorOps.cs:241-250).
 * The f32 entry points of that interface are kept below under their
 * original names; the quantised, device-resident entry points (si_*) are the
 * hot path: weights stay in HBM as GGUF K-quant blocks and are dequantised
 * inside the matvec/GEMM kernels.
 *
 * Conventions
 *  - Every si_* call returns an si_status (0 = SI_OK).  On failure the
 *    message is available from si_last_error() on the same thread.
 *  - Pointers named *_dev are device pointers of the context's GPU; pointers
 *    named *_host are host pointers, read or written before the call returns.
 *  - A context owns one CUDA stream.  Device-pointer calls are asynchronous
 *    on that stream; host-pointer calls synchronise before returning.  Calls
 *    on one context are not thread-safe; use one context per thread.
 *  - There is no CPU fallback: without a usable GPU, calls fail with
 *    SI_ERR_CUDA.
 */
#ifndef SHARPINFER_B200_H
#define SHARPINFER_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(_WIN32)
#define SI_EXPORT __declspec(dllexport)
#else
#define SI_EXPORT __attribute__((visibility("default")))
#endif

/* Status codes. */
typedef enum {
  SI_OK = 0,
  SI_ERR_INVALID = 1,     /* bad argument (null pointer, shape, type) */
  SI_ERR_CUDA = 2,        /* CUDA runtime error or no usable device */
  SI_ERR_OOM = 3,         /* device allocation failed */
  SI_ERR_UNSUPPORTED = 4, /* valid request this build does not implement */
  SI_ERR_NCCL = 5,        /* collective failure */
  SI_ERR_TIMEOUT = 6      /* a bounded device or host wait gave up */
} si_status;

/* GGML quantisation type ids, the values of SharpInfer's QuantType enum
 * (src/SharpInfer.Core/Tensors/Quantization.cs:6-22). */
typedef enum {
  SI_F32 = 0,
  SI_F16 = 1,
  SI_Q4_0 = 2,
  SI_Q8_0 = 8,
  SI_Q2_K = 10,
  SI_Q3_K = 11,
  SI_Q4_K = 12,
  SI_Q5_K = 13,
  SI_Q6_K = 14
} si_qtype;

/* Synthetic-data recipes for si_synth_* (benchmarks and tests). */
typedef enum {
  SI_SYNTH_PLAIN = 0, /* Q4_K: d,dmin=f16(|N|*sigma), 6-bit sc/m uniform 0..63 */
  SI_SYNTH_MODEL = 1  /* Q4_K: zero-mean weights, sc 1..8, m=round(7.5 sc), dmin=d */
} si_synth_recipe;

typedef struct si_ctx si_ctx;
typedef struct si_weight si_weight;

/* ---------------------------------------------------------------- lifecycle */

/* Library ABI version (major*10000 + minor*100 + patch). */
SI_EXPORT int si_version(void);

/* Message of the last failed call on this thread ("" if none). */
SI_EXPORT const char* si_last_error(void);

/* Bind a context to `device` and create its stream.  Replaces cuda_init
 * (src/SharpInfer.Gpu/Kernels/kernels.cu:30-37), which returned a null
 * handle on failure; here the reason is kept in si_last_error(). */
SI_EXPORT int si_init(int device, si_ctx** out);

/* Release the context's stream and scratch memory (cuda_cleanup, kernels.cu:39-43). */
SI_EXPORT int si_shutdown(si_ctx* ctx);

/* Device name into buf (NUL-terminated, truncated to len). */
SI_EXPORT int si_device_name(si_ctx* ctx, char* buf, int len);

/* The context's cudaStream_t, for callers that enqueue their own work. */
SI_EXPORT int si_stream(si_ctx* ctx, void** stream_out);

/* Wait for all work queued on the context's stream. */
SI_EXPORT int si_synchronize(si_ctx* ctx);

/* ------------------------------------------------------------------ weights */

/* Copy a row-major [rows][cols] tensor of raw GGUF blocks (cols/256 Q4_K or
 * Q6_K blocks, or cols/32 Q8_0 blocks per row) from host memory into a
 * device-resident weight.  The caller keeps ownership of `blocks_host`.
 * The bytes are what SharpInfer's loader hands to Dequantize.DequantizeTensor
 * (Quantization.cs:415-469); they are re-ordered on the device into the
 * kernel layout (same byte count) and never expanded to f32.  cols must be a
 * multiple of the block size.
 * Q4_0, Q2_K, Q3_K and Q5_K (cols a multiple of 256) are kept in their GGUF
 * block layout -- GGML's, as gguf-py decodes it: Q2_K [scales][qs][d][dmin],
 * Q3_K [hmask][qs][scales][d], Q5_K [d][dmin][scales][qh][qs] (the
 * reference's Quantization.cs:176-356 reads these three at other offsets) --
 * and serve si_dequant, si_qmatvec / si_qmatvec_host and si_qgemm. */
SI_EXPORT int si_weight_upload(si_ctx* ctx, int qtype, const void* blocks_host, int64_t rows,
                               int64_t cols, si_weight** out);

/* Generate a seeded synthetic weight directly on the device (benchmarks,
 * tests).  Bytes equal si_synth_blocks_host() for the same arguments. */
SI_EXPORT int si_weight_synth(si_ctx* ctx, int qtype, int64_t rows, int64_t cols, uint64_t seed,
                              uint64_t tag, int recipe, float sigma, si_weight** out);

SI_EXPORT int si_weight_free(si_weight* w);

/* Shape, type and device bytes of a weight (any out pointer may be NULL). */
SI_EXPORT int si_weight_info(const si_weight* w, int* qtype, int64_t* rows, int64_t* cols,
                             int64_t* device_bytes);

/* ---------------------------------------------------------------- host data */

/* Host-side generator of the same seeded blocks as si_weight_synth: fills
 * rows*cols/blocksize GGUF blocks into out_host (row-major). */
SI_EXPORT int si_synth_blocks_host(int qtype, int64_t rows, int64_t cols, uint64_t seed,
                                   uint64_t tag, int recipe, float sigma, void* out_host);

/* n f32 values mean + sigma*N(0,1) (seeded), host. */
SI_EXPORT int si_synth_f32_host(int64_t n, uint64_t seed, uint64_t tag, float mean, float sigma,
                                float* out_host);

/* n f16 values f16(sigma*N(0,1)) (seeded), host. */
SI_EXPORT int si_synth_f16_host(int64_t n, uint64_t seed, uint64_t tag, float sigma,
                                uint16_t* out_host);

/* -------------------------------------------------------------------- ops */

/* Dequantise a weight to f32 [rows][cols] in device memory, bit-exact with
 * Dequantize.DequantQ4_K / DequantQ6_K / DequantQ8_0
 * (Quantization.cs:273-314, 362-391, 106-114). */
SI_EXPORT int si_dequant(si_ctx* ctx, const si_weight* w, float* out_dev);

/* y[b][r] = sum_c W[r][c] * x[b][c] for b < batch (1..16), x [batch][cols]
 * f32, y [batch][rows] f32, both device pointers.  The quantised
 * counterpart of IComputeBackend.MatVecMul (TensorOps.cs:243, :63-72):
 * W is read once per call as K-quant blocks. */
SI_EXPORT int si_qmatvec(si_ctx* ctx, const si_weight* w, const float* x_dev, float* y_dev,
                         int batch);

/* Two-phase form of si_qmatvec for several weights that share an input:
 * si_act_prepare converts x [batch][cols] (device) once into the context's
 * activation staging (f16 hi/lo fragments, per-vector scale, Q4_K sub-block
 * sums); si_qmatvec_prepared then multiplies any weight with that many
 * columns.  accumulate != 0 adds into y instead of storing (residual add). */
SI_EXPORT int si_act_prepare(si_ctx* ctx, const float* x_dev, int64_t cols, int batch);
SI_EXPORT int si_qmatvec_prepared(si_ctx* ctx, const si_weight* w, float* y_dev, int batch,
                                  int accumulate);

/* Prefill GEMM: y[m][r] = sum_c W[r][c] * x[m][c] for m < M (any M >= 1),
 * x [M][cols] bf16 and y [M][rows] f32, both device pointers -- the batched
 * counterpart of IComputeBackend.MatMul (TensorOps.cs:244, :79-112) that
 * replaces the per-token prefill loop (InferenceEngine.cs:82-85).  W is
 * dequantised to f16 into context scratch, then multiplied on the tensor
 * cores (tcgen05, f32 accumulation); cols must be a multiple of 64. */
SI_EXPORT int si_qgemm(si_ctx* ctx, const si_weight* w, const uint16_t* x_bf16_dev, float* y_dev, int M);
/* Prefill attention on the tensor cores: FlashAttention.Forward
 * (src/SharpInfer.Core/Layers/FlashAttention.cs:59-167) for bf16 q [batch][heads][seq][128],
 * k, v [batch][kv_heads][kv][128] (grouped-query: head h reads kv head
 * h / (heads / kv_heads)), f32 o [batch][heads][seq][128], all device
 * pointers (16-byte aligned; k and v may be NULL when kv = 0).  causal != 0
 * lets query i see keys j <= i + start_pos; a query with no visible key gets
 * 0.  Runs on tcgen05 with S and O in tensor memory; v is transposed into
 * context scratch first.  Asynchronous on the context stream. */
SI_EXPORT int si_attn_prefill(si_ctx* ctx, const uint16_t* q_bf16, const uint16_t* k_bf16, const uint16_t* v_bf16,
                              float* o, int batch, int heads, int kv_heads, int seq, int kv, int head_dim, float scale,
                              int causal, int start_pos);

/* Keep a dequantised f16 copy of W (rows * cols * 2 bytes of device memory,
 * freed with the weight) so that later si_qgemm calls skip the dequantising
 * pass -- for prefill in several chunks over the same weights.  The copy is
 * what DequantizeTensor (Quantization.cs:415-469) produces, rounded to f16. */
SI_EXPORT int si_qgemm_cache_weight(si_ctx* ctx, si_weight* w);

/* Same with host buffers (copied in, computed, copied out, synchronised),
 * the calling convention of cuda_mat_vec_mul (kernels.cu:67-87). */
SI_EXPORT int si_qmatvec_host(si_ctx* ctx, const si_weight* w, const float* x_host,
                              float* y_host, int batch);

/* si_qmatvec for callers that cannot allocate device memory: no counterpart
 * in the reference.  It takes no context and calls no cudaMalloc/cudaFree.
 * Its scratch is one fixed 4 MiB array of device memory inside the library,
 * held by every GPU that loads the library until the process exits.
 * Limits: rows <= 32768, cols <= 16384, batch 1..16; larger shapes return
 * SI_ERR_UNSUPPORTED.  x [batch][cols] and y [batch][rows] are f32 device
 * pointers on w's device; `stream` is a cudaStream_t (NULL = legacy default
 * stream).  The call is synchronous on that stream.  Every call looks up the
 * array's device address (so a device reset between calls is harmless); the
 * first call on a device may load the library's kernels there, so make that
 * first call before any stream capture.  All calls on one GPU share the
 * array: calls whose work overlaps on the GPU (other streams or threads)
 * race -- serialise them. */
SI_EXPORT int si_qmatvec_noalloc(const si_weight* w, const float* x_dev, float* y_dev, int batch,
                                 void* stream);

/* ------------------------------------------------------------ decode model */

/* A Llama/Mistral-architecture model resident on one GPU: the forward pass of
 * Transformer.Forward (src/SharpInfer.Core/Layers/Transformer.cs:67-162) --
 * RmsNorm, Q/K/V projections, RoPE, KV store, GQA attention, O projection,
 * residual, RmsNorm, gate/up, SiLU*up, down, residual; final RmsNorm, lm_head
 * and greedy ArgMax (SamplingPipeline.cs:64-65) -- for `batch` sequences at
 * once, one token each, all at the same position.  Field names follow the
 * reference's ModelConfig (Transformer.cs:43-56, KVCache.cs:28-36). */
typedef struct {
  int n_layers;        /* NumLayers */
  int hidden;          /* HiddenSize */
  int intermediate;    /* IntermediateSize */
  int n_heads;         /* NumAttentionHeads */
  int n_kv_heads;      /* NumKvHeads */
  int head_dim;        /* HeadDim (128) */
  int vocab;           /* VocabSize */
  int max_seq;         /* KV positions per sequence (MaxSequenceLength) */
  int max_batch;       /* sequences decoded together (1..16) */
  float rms_eps;       /* RmsNormEps */
  float rope_theta;    /* RopeTheta */
  int weight_qtype;    /* projections: SI_Q4_K, SI_Q6_K or SI_Q8_0 */
  int lm_head_qtype;   /* OutputWeight */
  int emb_qtype;       /* TokenEmbedding (one row is dequantised per token) */
} si_model_config;

typedef struct si_model si_model;

/* Tensor ids for si_model_set_tensor / si_model_tensor_recipe. */
typedef enum {
  SI_T_Q = 0, SI_T_K = 1, SI_T_V = 2, SI_T_O = 3, SI_T_GATE = 4, SI_T_UP = 5, SI_T_DOWN = 6,
  SI_T_ATTN_NORM = 7, SI_T_FFN_NORM = 8,               /* layer >= 0 */
  SI_T_EMB = 100, SI_T_LM_HEAD = 101, SI_T_FINAL_NORM = 102 /* layer = -1 */
} si_tensor;

/* Allocate the model (weights, f16 KV cache, activations) on the context's
 * GPU.  Weights are undefined until set or synthesised. */
SI_EXPORT int si_model_create(si_ctx* ctx, const si_model_config* cfg, si_model** out);

/* ------------------------------------------------- tensor parallelism (TP)
 * The tensor-parallel path of InferenceCluster (src/SharpInfer.Core/Engine/
 * DistributedInference.cs:143-160) with the partial-sum exchange of its
 * AllReduce (:623-705) done on the GPUs, one rank per GPU: rank
 * `rank` of `tp` (1, 2, 4, 8) holds q/k/v heads, gate/up rows and lm_head
 * vocabulary rows 1/tp each (column-parallel), Wo / Wdown columns 1/tp each
 * (row-parallel), and its kv heads of the cache; the embedding and norms are
 * replicated.  After Wo and Wdown the ranks exchange partial sums directly in
 * each other's memory (NVLink peer stores, no collective library), and the
 * greedy token is chosen across the vocabulary slices.  Every rank runs the
 * same calls (set/synth, kv_synth, decode_step / decode_generate) in the same
 * order.  Logits returned by si_decode_step are this rank's slice
 * [batch][vocab / tp]. */
SI_EXPORT int si_model_create_tp(si_ctx* ctx, const si_model_config* cfg, int tp, int rank, si_model** out);
/* This rank's communication buffer as an IPC handle (len >= 64 bytes). */
SI_EXPORT int si_model_tp_handle(si_model* m, void* handle_out, int len);
/* Map every rank's buffer: handles of ranks 0 .. tp-1, 64 bytes each
 * (the handles of si_model_tp_handle, gathered by the host). */
SI_EXPORT int si_model_tp_connect(si_model* m, const void* handles, int len);
/* Connect ranks that live in one process (for example one host thread per
 * GPU) by their models instead of IPC handles: ranks[r] is rank r's model,
 * r = 0 .. tp-1, all of one configuration.  Peer access is enabled between
 * their devices.  Replaces the rank wiring of InferenceCluster
 * (DistributedInference.cs:33-160) for workers in one process.  A rank that
 * never steps makes the others' bounded waits give up -- the device-side
 * counterpart of WaitForResponseAsync's timeout (DistributedInference.cs:158,
 * :802): their si_decode_step returns SI_ERR_TIMEOUT after about a second
 * and the context stays usable. */
SI_EXPORT int si_model_tp_connect_local(si_model* m, si_model* const* ranks, int tp);
/* The part of a whole tensor a rank holds: global rows grow0 .. grow0 + rows,
 * and in each row quant blocks gb0 .. gb0 + nblk of gnblk.  No device work. */
SI_EXPORT int si_tp_slice(const si_model_config* cfg, int tp, int rank, int tensor, int64_t* grow0, int64_t* rows,
                          int64_t* gb0, int64_t* nblk, int64_t* gnblk);
SI_EXPORT int si_model_free(si_model* m);

/* The whole model's configuration (all ranks together for tensor parallelism). */
SI_EXPORT int si_model_get_config(const si_model* m, si_model_config* out);

/* Upload one weight tensor as raw GGUF blocks, row-major [rows][cols] of the
 * configured type (norms: f32[hidden]).  The projection shapes are those of
 * LayerWeights (Transformer.cs:89-151). */
SI_EXPORT int si_model_set_tensor(si_model* m, int layer, int tensor, const void* host);

/* Fill every weight and norm with the seeded synthetic recipe (benchmarks,
 * tests).  si_model_tensor_recipe reports, per tensor, the si_synth_* call
 * that reproduces its bytes on the host: generator tag, type, recipe, sigma
 * and shape (mean/sigma of the f32 norms in sigma/mean). */
SI_EXPORT int si_model_synth(si_model* m, uint64_t seed);
SI_EXPORT int si_model_tensor_recipe(const si_model_config* cfg, int layer, int tensor,
                                     uint64_t* tag, int* qtype, int* recipe, float* sigma,
                                     float* mean, int64_t* rows, int64_t* cols);

/* Fill cache positions [0, len) of every layer and sequence with f16 values
 * f16(N(0,1)) (seeded).  The K values of (layer l, sequence b) are
 * si_synth_f16_host(len*n_kv*head_dim, seed, si_model_kv_tag(l, b, 0), 1)
 * in the reference layout [pos][kv head][dim] (KVCache.cs:60-71). */
SI_EXPORT int si_model_kv_synth(si_model* m, int len, uint64_t seed);
SI_EXPORT uint64_t si_model_kv_tag(int layer, int seq, int is_value);

/* Write n cache positions from host f16 arrays in the reference layout
 * [n][kv head][dim] (KVCache.Store, KVCache.cs:46-57), all kv heads of the
 * model (a tensor-parallel rank keeps its own). */
SI_EXPORT int si_model_kv_write(si_model* m, int layer, int seq, int pos0, int n,
                                const uint16_t* k_host, const uint16_t* v_host);

/* One decode step: token ids tokens_host[batch] at position pos (the same for
 * every sequence; 0 <= pos < max_seq).  Writes the greedy next token of each
 * sequence to argmax_host[batch] and, if logits_host is not NULL, the logits
 * [batch][vocab].  Replayed as one CUDA graph per batch size. */
SI_EXPORT int si_decode_step(si_model* m, const int* tokens_host, int batch, int pos,
                             int* argmax_host, float* logits_host);

/* Greedy generation: nsteps decode steps from tokens_host[batch] at
 * positions pos0, pos0+1, ..., each step's argmax feeding the next step on
 * the device (the decode loop of InferenceEngine.GenerateAsync,
 * src/SharpInfer.Core/Engine/InferenceEngine.cs:96-131, with Temperature <= 0).
 * out_tokens_host[nsteps][batch] receives the generated tokens. */
SI_EXPORT int si_decode_generate(si_model* m, const int* tokens_host, int batch, int pos0,
                                 int nsteps, int* out_tokens_host);

/* Prefill: the n prompt tokens tokens_host[n] of sequence `seq` at positions
 * pos0 .. pos0 + n - 1 through every layer at once, storing their K/V in the
 * cache, and the greedy next token after the last one (argmax_host, may be
 * NULL) with its logits [vocab] (logits_host, may be NULL).  Replaces the
 * reference's prefill loop of one Transformer.Forward per prompt token
 * (src/SharpInfer.Core/Engine/InferenceEngine.cs:82-85): one tensor-core GEMM
 * per projection (si_qgemm's kernels, activations as f16 rows) and one causal
 * flash attention per layer on the cache's f16 K/V.  The stored K/V are the
 * values the decode step would store token by token.  Single-device models
 * only (tp = 1).  Synchronous. */
SI_EXPORT int si_model_prefill(si_model* m, int seq, const int* tokens_host, int n, int pos0, int* argmax_host,
                               float* logits_host);

/* Read cache positions pos0 .. pos0 + n - 1 of one layer and sequence as f16
 * in the reference layout [n][kv head][dim] (KVCache.GetKey / GetValue,
 * KVCache.cs:60-71). */
SI_EXPORT int si_model_kv_read(si_model* m, int layer, int seq, int pos0, int n, uint16_t* k_host, uint16_t* v_host);

/* Prompt-cache serialisation of positions 0 .. length - 1 of a sequence, in
 * the byte format of KVCache.WriteRawData / ReadRawData (KVCache.cs:84-114):
 * for each layer, K then V as f32 [length][kv heads * head_dim].  Export
 * widens the f16 cache exactly; import rounds to f16.  out_bytes / in_bytes
 * must be at least n_layers * 2 * length * n_kv_heads * head_dim * 4. */
SI_EXPORT int si_model_kv_export(si_model* m, int seq, int length, void* out_host, size_t out_bytes);
SI_EXPORT int si_model_kv_import(si_model* m, int seq, int length, const void* in_host, size_t in_bytes);

/* Kernel launches of one captured decode step at this batch size (captures
 * the step if needed): the device work behind one Transformer.Forward call
 * (Transformer.cs:67-162).  For measurement. */
SI_EXPORT int si_decode_step_kernels(si_model* m, int batch, int* kernels);

/* Attention of one layer alone (RoPE, KV append at pos, attention) for
 * qkv_dev [batch][(n_heads + 2 n_kv_heads) * head_dim] -> out_dev
 * [batch][n_heads * head_dim] (test hook for the attention kernel). */
SI_EXPORT int si_model_attention(si_model* m, int layer, const float* qkv_dev, float* out_dev,
                                 int batch, int pos);

/* ------------------------------------------------------------ GGUF files
 * The model loader behind InferenceEngine.Load (src/SharpInfer.Core/Engine/
 * InferenceEngine.cs:48-49), whose Models/ directory the reference does not
 * ship.  GGUF v2 and v3; the file is memory-mapped and its quantised blocks
 * go to the device unexpanded.  Type ids are ggml's (QuantType,
 * Quantization.cs:6-22). */
typedef struct si_gguf si_gguf;
SI_EXPORT int si_gguf_open(const char* path, si_gguf** out);
SI_EXPORT int si_gguf_close(si_gguf* g);
/* Format version, tensor and key/value counts, file offset of the data section. */
SI_EXPORT int si_gguf_info(const si_gguf* g, int* version, int64_t* n_tensors, int64_t* n_kv, int64_t* data_offset);
/* Metadata: integer (any integer or bool type), number (float or integer),
 * string (NUL-terminated, truncated to len), array item type and length. */
SI_EXPORT int si_gguf_meta_int(const si_gguf* g, const char* key, int64_t* out);
SI_EXPORT int si_gguf_meta_float(const si_gguf* g, const char* key, double* out);
SI_EXPORT int si_gguf_meta_string(const si_gguf* g, const char* key, char* buf, int len);
SI_EXPORT int si_gguf_meta_array(const si_gguf* g, const char* key, int* item_type, int64_t* count);
/* Tensor i: name, ggml type, rows (product of the outer dimensions), cols
 * (the innermost dimension) and bytes; its bytes in the mapped file. */
SI_EXPORT int si_gguf_tensor_info(const si_gguf* g, int64_t i, char* name, int name_len, int* qtype, int64_t* rows,
                                  int64_t* cols, int64_t* bytes);
SI_EXPORT int si_gguf_find_tensor(const si_gguf* g, const char* name, int64_t* index);
SI_EXPORT int si_gguf_tensor_data(const si_gguf* g, int64_t i, const void** data);
/* The si_model_config of a llama/mistral-architecture file (general.
 * architecture and its block_count, embedding_length, feed_forward_length,
 * attention.head_count[_kv], attention.key_length, layer_norm_rms_epsilon,
 * rope.freq_base; vocabulary from token_embd).  max_seq <= 0 takes the
 * file's context_length.  The projections must all be one of Q4_K, Q6_K,
 * Q8_0 (SI_ERR_UNSUPPORTED names the first that is not). */
SI_EXPORT int si_gguf_model_config(const si_gguf* g, int max_seq, int max_batch, si_model_config* cfg);
/* Upload every tensor of the file into a model created with its config
 * (any tensor-parallel rank takes its own slices); a file without
 * output.weight uses the embedding as lm_head (tied weights). */
SI_EXPORT int si_model_load_gguf(si_model* m, const si_gguf* g);

/* --------------------------------------------- f32 interface of CudaBackend
 * The functions SharpInfer's managed backend binds from `sharpinfer_cuda`
 * (src/SharpInfer.Gpu/CudaBackend.cs:141-163), with the same signatures and
 * conventions: void returns (failures go to si_last_error() only), host
 * pointers valid for the call (device pointers also accepted), synchronous.
 * Operators follow TensorOps.cs. */

/* CudaBackend.cs:143 -- a handle (si_ctx*) or NULL when no B200 is usable. */
SI_EXPORT void* cuda_init(int device_id);
/* CudaBackend.cs:144 */
SI_EXPORT void cuda_cleanup(void* handle);
/* CudaBackend.cs:145 -- NUL-terminated device name into buffer[buf_len]. */
SI_EXPORT void cuda_device_name(void* handle, char* buffer, int buf_len);
/* HardwareBackends.cs:440 (CudaProbe.cuda_is_available): 1 if a CUDA device exists. */
SI_EXPORT int cuda_is_available(void);
/* HardwareBackends.cs:441 binds a zero-argument `cuda_device_name`, which
 * cannot share its name with the three-argument export above; this is that
 * probe under its own name (device 0; a per-thread buffer). */
SI_EXPORT const char* cuda_device_name_str(void);
/* CudaBackend.cs:147-148 -- result[r] = Dot(mat[r, :], vec) (TensorOps.cs:63-72). */
SI_EXPORT void cuda_mat_vec_mul(void* handle, const float* mat, const float* vec, float* result, int rows,
                                int cols);
/* CudaBackend.cs:150-151 -- C[M][N] = A[M][K] B[K][N] (TensorOps.cs:79-112). */
SI_EXPORT void cuda_mat_mul(void* handle, const float* a, const float* b, float* c, int M, int K, int N);
/* CudaBackend.cs:153-154 -- softmax in place (TensorOps.cs:115-132). */
SI_EXPORT void cuda_softmax(void* handle, float* x, int len);
/* CudaBackend.cs:156-157 -- output = RmsNorm(x) * weight (TensorOps.cs:135-145). */
SI_EXPORT void cuda_rms_norm(void* handle, float* output, const float* x, const float* weight, int size,
                             float eps);
/* CudaBackend.cs:159-160 -- x = SiLU(x) (TensorOps.cs:191-195). */
SI_EXPORT void cuda_silu(void* handle, float* x, int len);
/* CudaBackend.cs:162-163 -- a += b (TensorOps.cs:149-165). */
SI_EXPORT void cuda_add_inplace(void* handle, float* a, const float* b, int len);
/* Layers/FlashAttention.cs:380-384 (NativeFlashAttn, Cdecl): f32 Q, O [batch][heads][seq][head_dim],
 * K, V [batch][heads][kv][head_dim]; causal masking lets query i see keys
 * j <= i + (kv - seq); head_dim <= 256.  Semantics of FlashAttention.Forward
 * (FlashAttention.cs:59-167). */
SI_EXPORT void flash_attention_forward(void* Q, void* K, void* V, void* O, int batch, int heads, int seq, int kv,
                                       int head_dim, float scale, int causal);

#ifdef __cplusplus
}
#endif

#endif /* SHARPINFER_B200_H */
