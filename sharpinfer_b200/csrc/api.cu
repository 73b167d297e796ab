// C ABI: contexts, errors, weights, synthetic data and the quantised matvec.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <thread>
#include <vector>

#include "common.cuh"
#include "synth.h"

namespace si {

static thread_local char g_err[1024];

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

void clear_error() { g_err[0] = 0; }

int bind_device(si_ctx* c) {
  SI_CUDA(cudaSetDevice(c->device));
  return SI_OK;
}

int ensure(si_devbuf& b, size_t bytes) {
  if (b.bytes >= bytes && b.ptr) return SI_OK;
  if (b.ptr) cudaFree(b.ptr);
  b.ptr = nullptr;
  b.bytes = 0;
  size_t want = std::max(bytes, (size_t)4096);
  cudaError_t e = cudaMalloc(&b.ptr, want);
  if (e != cudaSuccess) {
    b.ptr = nullptr;
    SI_FAIL(e == cudaErrorMemoryAllocation ? SI_ERR_OOM : SI_ERR_CUDA,
            "cudaMalloc(%zu) failed: %s", want, cudaGetErrorString(e));
  }
  b.bytes = want;
  return SI_OK;
}

int ensure_pinned(si_ctx* c, size_t bytes) {
  if (c->pinned_bytes >= bytes && c->pinned) return SI_OK;
  if (c->pinned) cudaFreeHost(c->pinned);
  c->pinned = nullptr;
  c->pinned_bytes = 0;
  size_t want = std::max(bytes, (size_t)65536);
  SI_CUDA(cudaMallocHost(&c->pinned, want));
  c->pinned_bytes = want;
  return SI_OK;
}

static int check_qtype(int qt) {
  if (qt != SI_Q4_K && qt != SI_Q6_K && qt != SI_Q8_0 && !raw_layout(qt))
    SI_FAIL(SI_ERR_UNSUPPORTED,
            "quant type %d is not one of Q4_0(2), Q8_0(8), Q2_K(10), Q3_K(11), Q4_K(12), Q5_K(13), Q6_K(14)", qt);
  return SI_OK;
}

static int check_shape(int qt, int64_t rows, int64_t cols) {
  if (rows <= 0 || cols <= 0) SI_FAIL(SI_ERR_INVALID, "weight shape %lldx%lld must be positive",
                                      (long long)rows, (long long)cols);
  const int unit = raw_layout(qt) ? 256 : block_elems(qt);  // raw formats: 256-element units
  if (cols % unit)
    SI_FAIL(SI_ERR_INVALID, "cols=%lld is not a multiple of %d", (long long)cols, unit);
  if (cols > SI_MAX_K) SI_FAIL(SI_ERR_INVALID, "cols=%lld above the supported maximum %d",
                               (long long)cols, SI_MAX_K);
  if (rows > (int64_t)1 << 31) SI_FAIL(SI_ERR_INVALID, "rows=%lld too large", (long long)rows);
  return SI_OK;
}

static int weight_alloc(si_ctx* c, int qt, int64_t rows, int64_t cols, si_weight** out) {
  SI_TRY(check_qtype(qt));
  SI_TRY(check_shape(qt, rows, cols));
  si_weight* w = new si_weight();
  w->qtype = qt;
  w->rows = rows;
  w->cols = cols;
  w->tiles = (rows + 15) / 16;
  w->nblk = cols / block_elems(qt);
  w->bytes = raw_layout(qt) ? (size_t)(rows * w->nblk * gguf_block_bytes(qt))
                            : (size_t)(w->tiles * w->nblk * tile_block_bytes(qt));
  w->device = c->device;
  cudaError_t e = cudaMalloc(&w->dev, w->bytes);
  if (e != cudaSuccess) {
    size_t bytes = w->bytes;
    delete w;
    SI_FAIL(e == cudaErrorMemoryAllocation ? SI_ERR_OOM : SI_ERR_CUDA,
            "weight allocation of %zu bytes failed: %s", bytes, cudaGetErrorString(e));
  }
  *out = w;
  return SI_OK;
}

// Read and clear the device error word after the stream has been synchronised.
int check_device_errors(si_ctx* c) {
  int v = 0;
  SI_CUDA(cudaMemcpy(&v, c->dev_err, sizeof(int), cudaMemcpyDeviceToHost));
  if (v) {
    // a kernel gave up part-way: clear the error word and the shared-tile counters
    SI_CUDA(cudaMemset(c->dev_err, 0, sizeof(int)));
    if (c->qmv_count.ptr) SI_CUDA(cudaMemset(c->qmv_count.ptr, 0, c->qmv_count.bytes));
    SI_FAIL(SI_ERR_TIMEOUT, "a device-side bounded wait gave up (error bits 0x%x)", v);
  }
  return SI_OK;
}

// Grow the streaming-matvec scratch for weight w (counters start at zero).
int ensure_qmv_scratch(si_ctx* c, const si_weight* w) {
  size_t sb;
  int64_t cn;
  const int64_t nunit = w->qtype == SI_Q8_0 ? (w->nblk + 7) / 8 : w->nblk;
  qmv_scratch_need(w->tiles, nunit, c->sm_count, &sb, &cn);
  if (c->qmv_split.bytes < sb) SI_TRY(ensure(c->qmv_split, sb));
  if (c->qmv_count.bytes < (size_t)cn * 4) {
    SI_TRY(ensure(c->qmv_count, (size_t)cn * 4));
    SI_CUDA(cudaMemset(c->qmv_count.ptr, 0, c->qmv_count.bytes));
  }
  return SI_OK;
}

// Row chunk (multiple of 16 rows) whose GGUF bytes fit the staging budget.
static int64_t chunk_rows(int qt, int64_t cols) {
  const int64_t budget = 64ll << 20;
  int64_t rb = (cols / block_elems(qt)) * gguf_block_bytes(qt);
  int64_t r = std::max<int64_t>(16, (budget / rb) / 16 * 16);
  return r;
}

}  // namespace si

using namespace si;

extern "C" {

SI_EXPORT int si_version(void) { return 100; }

SI_EXPORT const char* si_last_error(void) { return g_err; }

SI_EXPORT int si_init(int device, si_ctx** out) {
  clear_error();
  if (!out) SI_FAIL(SI_ERR_INVALID, "si_init: out is NULL");
  *out = nullptr;
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n == 0)
    SI_FAIL(SI_ERR_CUDA, "no CUDA device available (%s)", e != cudaSuccess ? cudaGetErrorString(e) : "0 devices");
  if (device < 0 || device >= n) SI_FAIL(SI_ERR_INVALID, "device %d out of range [0, %d)", device, n);
  SI_CUDA(cudaSetDevice(device));
  cudaDeviceProp prop;
  SI_CUDA(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10)
    SI_FAIL(SI_ERR_UNSUPPORTED, "device %d (%s, sm_%d%d) is not sm_100; this build targets B200",
            device, prop.name, prop.major, prop.minor);
  si_ctx* c = new si_ctx();
  c->device = device;
  c->sm_count = prop.multiProcessorCount;
  c->l2_bytes = prop.l2CacheSize;
  e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    delete c;
    SI_FAIL(SI_ERR_CUDA, "cudaStreamCreate failed: %s", cudaGetErrorString(e));
  }
  e = cudaMalloc(&c->dev_err, sizeof(int));
  if (e == cudaSuccess) e = cudaMemset(c->dev_err, 0, sizeof(int));

  if (e != cudaSuccess) {
    cudaStreamDestroy(c->stream);
    delete c;
    SI_FAIL(SI_ERR_CUDA, "context allocation failed: %s", cudaGetErrorString(e));
  }
  *out = c;
  return SI_OK;
}

SI_EXPORT int si_shutdown(si_ctx* c) {
  clear_error();
  if (!c) return SI_OK;
  cudaSetDevice(c->device);
  cudaStreamSynchronize(c->stream);
  for (si_devbuf* b : {&c->xprep, &c->stage[0], &c->stage[1], &c->stage[2], &c->stage[3]})
    if (b->ptr) cudaFree(b->ptr);
  if (c->pinned) cudaFreeHost(c->pinned);
  if (c->dev_err) cudaFree(c->dev_err);
  if (c->qmv_split.ptr) cudaFree(c->qmv_split.ptr);
  if (c->qmv_count.ptr) cudaFree(c->qmv_count.ptr);
  cudaStreamDestroy(c->stream);
  delete c;
  return SI_OK;
}

SI_EXPORT int si_device_name(si_ctx* c, char* buf, int len) {
  clear_error();
  if (!c || !buf || len <= 0) SI_FAIL(SI_ERR_INVALID, "si_device_name: bad arguments");
  cudaDeviceProp prop;
  SI_CUDA(cudaGetDeviceProperties(&prop, c->device));
  strncpy(buf, prop.name, (size_t)len - 1);
  buf[len - 1] = 0;
  return SI_OK;
}

SI_EXPORT int si_stream(si_ctx* c, void** s) {
  clear_error();
  if (!c || !s) SI_FAIL(SI_ERR_INVALID, "si_stream: bad arguments");
  *s = (void*)c->stream;
  return SI_OK;
}

SI_EXPORT int si_synchronize(si_ctx* c) {
  clear_error();
  if (!c) SI_FAIL(SI_ERR_INVALID, "si_synchronize: ctx is NULL");
  SI_TRY(bind_device(c));
  SI_CUDA(cudaStreamSynchronize(c->stream));
  return check_device_errors(c);
}

SI_EXPORT int si_weight_upload(si_ctx* c, int qt, const void* blocks, int64_t rows, int64_t cols,
                               si_weight** out) {
  clear_error();
  if (!c || !blocks || !out) SI_FAIL(SI_ERR_INVALID, "si_weight_upload: NULL argument");
  *out = nullptr;
  SI_TRY(bind_device(c));
  si_weight* w = nullptr;
  SI_TRY(weight_alloc(c, qt, rows, cols, &w));
  const int64_t rb = w->nblk * gguf_block_bytes(qt);
  const int64_t cr = chunk_rows(qt, cols);
  int st = ensure(c->stage[0], (size_t)(cr * rb));
  for (int64_t r0 = 0; st == SI_OK && r0 < rows; r0 += cr) {
    int64_t nr = std::min(cr, rows - r0);
    cudaError_t e = cudaMemcpyAsync(c->stage[0].ptr, (const uint8_t*)blocks + r0 * rb,
                                    (size_t)(nr * rb), cudaMemcpyHostToDevice, c->stream);
    if (e != cudaSuccess) {
      set_error("weight upload copy failed: %s", cudaGetErrorString(e));
      st = SI_ERR_CUDA;
      break;
    }
    if (raw_layout(qt)) {  // kept as GGUF blocks
      e = cudaMemcpyAsync((uint8_t*)w->dev + r0 * rb, c->stage[0].ptr, (size_t)(nr * rb), cudaMemcpyDeviceToDevice,
                          c->stream);
      if (e != cudaSuccess) {
        set_error("weight upload copy failed: %s", cudaGetErrorString(e));
        st = SI_ERR_CUDA;
      }
    } else {
      st = launch_repack(c, qt, (const uint8_t*)c->stage[0].ptr, rows, cols, r0, nr, w->dev);
    }
    if (st == SI_OK) {
      e = cudaStreamSynchronize(c->stream);  // staging is reused by the next chunk
      if (e != cudaSuccess) {
        set_error("weight repack failed: %s", cudaGetErrorString(e));
        st = SI_ERR_CUDA;
      }
    }
  }
  if (st != SI_OK) {
    cudaFree(w->dev);
    delete w;
    return st;
  }
  *out = w;
  return SI_OK;
}

SI_EXPORT int si_weight_synth(si_ctx* c, int qt, int64_t rows, int64_t cols, uint64_t seed,
                              uint64_t tag, int recipe, float sigma, si_weight** out) {
  clear_error();
  if (!c || !out) SI_FAIL(SI_ERR_INVALID, "si_weight_synth: NULL argument");
  *out = nullptr;
  SI_TRY(bind_device(c));
  if (raw_layout(qt)) SI_FAIL(SI_ERR_UNSUPPORTED, "si_weight_synth: no generator for quant type %d", qt);
  si_weight* w = nullptr;
  SI_TRY(weight_alloc(c, qt, rows, cols, &w));
  const int64_t rb = w->nblk * gguf_block_bytes(qt);
  const int64_t cr = chunk_rows(qt, cols);
  int st = ensure(c->stage[0], (size_t)(cr * rb));
  for (int64_t r0 = 0; st == SI_OK && r0 < rows; r0 += cr) {
    int64_t nr = std::min(cr, rows - r0);
    st = launch_synth_blocks(c, qt, seed, tag, recipe, sigma, r0 * w->nblk, nr * w->nblk,
                             (uint8_t*)c->stage[0].ptr);
    if (st == SI_OK) st = launch_repack(c, qt, (const uint8_t*)c->stage[0].ptr, rows, cols, r0, nr, w->dev);
    if (st == SI_OK) {
      cudaError_t e = cudaStreamSynchronize(c->stream);
      if (e != cudaSuccess) {
        set_error("synthetic weight generation failed: %s", cudaGetErrorString(e));
        st = SI_ERR_CUDA;
      }
    }
  }
  if (st != SI_OK) {
    cudaFree(w->dev);
    delete w;
    return st;
  }
  *out = w;
  return SI_OK;
}

SI_EXPORT int si_weight_free(si_weight* w) {
  clear_error();
  if (!w) return SI_OK;
  cudaSetDevice(w->device);
  if (w->dev) cudaFree(w->dev);
  if (w->f16) cudaFree(w->f16);
  delete w;
  return SI_OK;
}

SI_EXPORT int si_weight_info(const si_weight* w, int* qt, int64_t* rows, int64_t* cols,
                             int64_t* bytes) {
  clear_error();
  if (!w) SI_FAIL(SI_ERR_INVALID, "si_weight_info: weight is NULL");
  if (qt) *qt = w->qtype;
  if (rows) *rows = w->rows;
  if (cols) *cols = w->cols;
  if (bytes) *bytes = (int64_t)w->bytes;
  return SI_OK;
}

SI_EXPORT int si_synth_blocks_host(int qt, int64_t rows, int64_t cols, uint64_t seed, uint64_t tag,
                                   int recipe, float sigma, void* out) {
  clear_error();
  if (!out) SI_FAIL(SI_ERR_INVALID, "si_synth_blocks_host: out is NULL");
  SI_TRY(check_qtype(qt));
  if (raw_layout(qt)) SI_FAIL(SI_ERR_UNSUPPORTED, "si_synth_blocks_host: no generator for quant type %d", qt);
  if (rows <= 0 || cols <= 0 || cols % block_elems(qt))
    SI_FAIL(SI_ERR_INVALID, "bad synthetic shape %lldx%lld", (long long)rows, (long long)cols);
  const uint64_t key = si_key(seed, tag);
  const int64_t nb = rows * (cols / block_elems(qt));
  const int bb = gguf_block_bytes(qt);
  uint8_t* dst = (uint8_t*)out;
  unsigned nt = std::max(1u, std::min(32u, std::thread::hardware_concurrency()));
  std::vector<std::thread> th;
  for (unsigned k = 0; k < nt; k++) {
    th.emplace_back([=]() {
      int64_t lo = nb * k / nt, hi = nb * (k + 1) / nt;
      for (int64_t i = lo; i < hi; i++) {
        if (qt == SI_Q4_K) si_synth_q4k_block(key, (uint64_t)i, sigma, recipe, dst + i * bb);
        else if (qt == SI_Q6_K) si_synth_q6k_block(key, (uint64_t)i, sigma, dst + i * bb);
        else si_synth_q80_block(key, (uint64_t)i, sigma, dst + i * bb);
      }
    });
  }
  for (auto& t : th) t.join();
  return SI_OK;
}

SI_EXPORT int si_synth_f32_host(int64_t n, uint64_t seed, uint64_t tag, float mean, float sigma,
                                float* out) {
  clear_error();
  if (!out || n < 0) SI_FAIL(SI_ERR_INVALID, "si_synth_f32_host: bad arguments");
  const uint64_t key = si_key(seed, tag);
  for (int64_t i = 0; i < n; i++) out[i] = si_synth_f32(key, (uint64_t)i, mean, sigma);
  return SI_OK;
}

SI_EXPORT int si_synth_f16_host(int64_t n, uint64_t seed, uint64_t tag, float sigma, uint16_t* out) {
  clear_error();
  if (!out || n < 0) SI_FAIL(SI_ERR_INVALID, "si_synth_f16_host: bad arguments");
  const uint64_t key = si_key(seed, tag);
  unsigned nt = std::max(1u, std::min(32u, std::thread::hardware_concurrency()));
  std::vector<std::thread> th;
  for (unsigned k = 0; k < nt; k++) {
    th.emplace_back([=]() {
      int64_t lo = n * k / nt, hi = n * (k + 1) / nt;
      for (int64_t i = lo; i < hi; i++) out[i] = si_synth_f16(key, (uint64_t)i, sigma);
    });
  }
  for (auto& t : th) t.join();
  return SI_OK;
}

SI_EXPORT int si_dequant(si_ctx* c, const si_weight* w, float* out) {
  clear_error();
  if (!c || !w || !out) SI_FAIL(SI_ERR_INVALID, "si_dequant: NULL argument");
  if (w->device != c->device) SI_FAIL(SI_ERR_INVALID, "si_dequant: weight lives on device %d, context on %d", w->device, c->device);
  SI_TRY(bind_device(c));
  if (raw_layout(w->qtype)) return launch_dequant_raw(c->stream, w, out);
  return launch_dequant(c, w, out);
}

SI_EXPORT int si_act_prepare(si_ctx* c, const float* x, int64_t cols, int batch) {
  clear_error();
  if (!c || !x) SI_FAIL(SI_ERR_INVALID, "si_act_prepare: NULL argument");
  if (batch < 1 || batch > SI_MAX_BATCH) SI_FAIL(SI_ERR_INVALID, "si_act_prepare: batch %d outside 1..%d", batch, SI_MAX_BATCH);
  if (cols <= 0 || cols % 32 || cols > SI_MAX_K)
    SI_FAIL(SI_ERR_INVALID, "si_act_prepare: cols=%lld must be a multiple of 32 in [32, %d]", (long long)cols, SI_MAX_K);
  SI_TRY(bind_device(c));
  const int K = (int)cols;
  SI_TRY(ensure(c->xprep, xprep_bytes(K, batch)));
  SI_TRY(launch_prep(c->stream, x, K, nullptr, nullptr, 0.f, SI_PREP_PLAIN, K, batch, nullptr,
                     (uint8_t*)c->xprep.ptr, false));
  c->prep_cols = K;
  c->prep_batch = batch;
  return SI_OK;
}

SI_EXPORT int si_qmatvec_prepared(si_ctx* c, const si_weight* w, float* y, int batch, int accumulate) {
  clear_error();
  if (!c || !w || !y) SI_FAIL(SI_ERR_INVALID, "si_qmatvec_prepared: NULL argument");
  if (w->device != c->device) SI_FAIL(SI_ERR_INVALID, "si_qmatvec: weight lives on device %d, context on %d", w->device, c->device);
  if (raw_layout(w->qtype))
    SI_FAIL(SI_ERR_UNSUPPORTED, "si_qmatvec_prepared: quant type %d multiplies f32 activations (si_qmatvec)",
            w->qtype);
  if (c->prep_cols != w->cols || c->prep_batch != batch)
    SI_FAIL(SI_ERR_INVALID, "si_qmatvec_prepared: prepared activations are %dx%d, weight needs %dx%lld",
            c->prep_batch, c->prep_cols, batch, (long long)w->cols);
  SI_TRY(bind_device(c));
  SI_TRY(ensure_qmv_scratch(c, w));
  return launch_qmv(c->stream, w, (const uint8_t*)c->xprep.ptr, batch, y,
                    accumulate ? SI_EPI_ADD : SI_EPI_STORE, c->qmv(), true);
}

SI_EXPORT int si_qmatvec(si_ctx* c, const si_weight* w, const float* x, float* y, int batch) {
  clear_error();
  if (!c || !w || !x || !y) SI_FAIL(SI_ERR_INVALID, "si_qmatvec: NULL argument");
  if (batch < 1 || batch > SI_MAX_BATCH) SI_FAIL(SI_ERR_INVALID, "si_qmatvec: batch %d outside 1..%d", batch, SI_MAX_BATCH);
  if (raw_layout(w->qtype)) {
    if (w->device != c->device) SI_FAIL(SI_ERR_INVALID, "si_qmatvec: weight lives on device %d, context on %d",
                                        w->device, c->device);
    SI_TRY(bind_device(c));
    return launch_qmv_raw(c->stream, w, x, y, batch);
  }
  SI_TRY(si_act_prepare(c, x, w->cols, batch));
  return si_qmatvec_prepared(c, w, y, batch, 0);
}

SI_EXPORT int si_qmatvec_host(si_ctx* c, const si_weight* w, const float* x, float* y, int batch) {
  clear_error();
  if (!c || !w || !x || !y) SI_FAIL(SI_ERR_INVALID, "si_qmatvec_host: NULL argument");
  if (batch < 1 || batch > SI_MAX_BATCH) SI_FAIL(SI_ERR_INVALID, "si_qmatvec_host: batch %d outside 1..%d", batch, SI_MAX_BATCH);
  SI_TRY(bind_device(c));
  const size_t xb = (size_t)batch * w->cols * 4, yb = (size_t)batch * w->rows * 4;
  SI_TRY(ensure(c->stage[1], xb));
  SI_TRY(ensure(c->stage[2], yb));
  SI_TRY(ensure_pinned(c, xb + yb));
  memcpy(c->pinned, x, xb);
  SI_CUDA(cudaMemcpyAsync(c->stage[1].ptr, c->pinned, xb, cudaMemcpyHostToDevice, c->stream));
  SI_TRY(si_qmatvec(c, w, (const float*)c->stage[1].ptr, (float*)c->stage[2].ptr, batch));
  uint8_t* yh = (uint8_t*)c->pinned + xb;
  SI_CUDA(cudaMemcpyAsync(yh, c->stage[2].ptr, yb, cudaMemcpyDeviceToHost, c->stream));
  SI_CUDA(cudaStreamSynchronize(c->stream));
  SI_TRY(check_device_errors(c));
  memcpy(y, yh, yb);
  return SI_OK;
}

}  // extern "C"
