// si_qmatvec_noalloc: the quantised matvec for callers that must not allocate
// device memory.
//
// Who needs it: a host that has handed all of a GPU's free memory to its own
// pool (an engine that sizes its KV cache to fill HBM, or a process running
// under a hard device-memory budget) cannot let a library call cudaMalloc.
// Nor can a latency-critical caller that must never meet the device-wide
// synchronisation cudaMalloc/cudaFree imply.  si_qmatvec grows a per-context
// scratch on demand; this entry point needs no context and allocates nothing.
//
// Its scratch is one fixed array in this module, kNoAllocScratchBytes (4 MiB)
// of device memory that every GPU which loads the library holds until the
// process exits.  It is shared by every call on that GPU, so two calls whose
// kernels overlap on the GPU (different streams, or different host threads)
// race on it and may both return wrong results: serialise them.
//
// Layout of the array (offsets in bytes):
//   [0, 256)           device error word          -- cleared by every call
//   [256, 8448)        per-row-tile arrival counts -- cleared by every call
//   [8448, +X)         prepared activations (X = 1,085,440 B at most)
//   [256-aligned, end) partial sums of row tiles split between warps
// Only the error word and the counters must start at zero; every call clears
// them on its stream before its kernels run.
//
// Limits: rows <= 32768, cols <= 16384, batch <= 16.  Larger shapes are
// rejected with SI_ERR_UNSUPPORTED before anything is launched.
#include <mutex>

#include "common.cuh"

namespace si {
namespace {

constexpr size_t kNoAllocScratchBytes = 4u << 20;
constexpr size_t kErrOff = 0, kCountOff = 256, kCountInts = 2048, kPrepOff = 256 + 4 * kCountInts;
constexpr int64_t kMaxRows = 32768, kMaxCols = 16384;
constexpr int kMaxDevices = 64;

static_assert(kMaxRows / 16 <= (int64_t)kCountInts, "one counter per row tile");
static_assert(kPrepOff % 256 == 0, "prepared activations start 256-byte aligned");

// The scratch.  In host code `g_noalloc_scratch` names a host-side stand-in
// for this symbol, not device memory: its device address comes only from
// cudaGetSymbolAddress, made per device with that device current.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

struct DeviceScratch {
  uint8_t* base = nullptr;  // device address of g_noalloc_scratch on this device
  int sms = 0;
};

std::mutex g_setup_mu;
int g_sms[kMaxDevices];  // SM count per device, 0 until first asked

// With `dev` current: the array's device address and the SM count.  The
// address is looked up on every call (a cheap runtime query), so it stays
// right when the caller has reset the device or rebuilt its primary context
// between calls.  The first lookup on a device may load the module there, so
// the first call on a device must not happen during stream capture.
int scratch_for(int dev, DeviceScratch* out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess)
    SI_FAIL(SI_ERR_CUDA, "si_qmatvec_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
            cudaGetErrorString(e));
  out->base = (uint8_t*)p;
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (!g_sms[dev]) {
    int sms = 0;
    SI_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    g_sms[dev] = sms;
  }
  out->sms = g_sms[dev];
  return SI_OK;
}

int run(const si_weight* w, const float* x, float* y, int batch, cudaStream_t s, int dev) {
  if (raw_layout(w->qtype)) {  // GGUF-layout formats need no scratch at all
    SI_TRY(launch_qmv_raw(s, w, x, y, batch));
    SI_CUDA(cudaStreamSynchronize(s));
    return SI_OK;
  }
  DeviceScratch sc;
  SI_TRY(scratch_for(dev, &sc));
  const int K = (int)w->cols;
  const size_t split_off = (kPrepOff + xprep_bytes(K, batch) + 255) & ~(size_t)255;
  const int64_t nunit = w->qtype == SI_Q8_0 ? (w->nblk + 7) / 8 : w->nblk;
  size_t split_need;
  int64_t counts;
  qmv_scratch_need(w->tiles, nunit, sc.sms, &split_need, &counts, false);
  if (split_off + split_need > kNoAllocScratchBytes || counts > (int64_t)kCountInts)
    SI_FAIL(SI_ERR_UNSUPPORTED, "si_qmatvec_noalloc: %lldx%lld at batch %d needs %zu bytes of scratch, %zu available",
            (long long)w->rows, (long long)w->cols, batch, split_off + split_need, kNoAllocScratchBytes);
  uint8_t* base = sc.base;
  int* err = (int*)(base + kErrOff);
  SI_CUDA(cudaMemsetAsync(base, 0, kPrepOff, s));  // error word + counters
  uint8_t* xprep = base + kPrepOff;
  SI_TRY(launch_prep(s, x, K, nullptr, nullptr, 0.f, SI_PREP_PLAIN, K, batch, nullptr, xprep, false));
  QmvBuffers qb;
  qb.split = (float*)(base + split_off);
  qb.split_bytes = kNoAllocScratchBytes - split_off;
  qb.count = (int*)(base + kCountOff);
  qb.count_n = (int64_t)kCountInts;
  qb.err = err;
  qb.sms = sc.sms;
  SI_TRY(launch_qmv(s, w, xprep, batch, y, SI_EPI_STORE, qb, false));
  // Synchronous, like the reference's calls: report a device-side wait that
  // gave up (the kernels then leave y incomplete).
  int v = 0;
  SI_CUDA(cudaMemcpyAsync(&v, err, sizeof(int), cudaMemcpyDeviceToHost, s));
  SI_CUDA(cudaStreamSynchronize(s));
  if (v) SI_FAIL(SI_ERR_TIMEOUT, "si_qmatvec_noalloc: a device-side bounded wait gave up (0x%x)", v);
  return SI_OK;
}

}  // namespace
}  // namespace si

using namespace si;

extern "C" SI_EXPORT int si_qmatvec_noalloc(const si_weight* w, const float* x_dev, float* y_dev, int batch,
                                            void* stream) {
  clear_error();
  if (!w || !x_dev || !y_dev) SI_FAIL(SI_ERR_INVALID, "si_qmatvec_noalloc: NULL argument");
  if (batch < 1 || batch > SI_MAX_BATCH)
    SI_FAIL(SI_ERR_INVALID, "si_qmatvec_noalloc: batch %d outside 1..%d", batch, SI_MAX_BATCH);
  if (w->rows > kMaxRows || w->cols > kMaxCols)
    SI_FAIL(SI_ERR_UNSUPPORTED, "si_qmatvec_noalloc: %lldx%lld weight above the limit of %lld rows x %lld cols",
            (long long)w->rows, (long long)w->cols, (long long)kMaxRows, (long long)kMaxCols);
  if (w->device < 0 || w->device >= kMaxDevices)
    SI_FAIL(SI_ERR_UNSUPPORTED, "si_qmatvec_noalloc: device %d above %d", w->device, kMaxDevices - 1);
  int prev = 0;
  SI_CUDA(cudaGetDevice(&prev));
  if (prev != w->device) SI_CUDA(cudaSetDevice(w->device));
  const int st = run(w, x_dev, y_dev, batch, (cudaStream_t)stream, w->device);
  if (prev != w->device) cudaSetDevice(prev);
  return st;
}
