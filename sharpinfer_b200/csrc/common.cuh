// Shared definitions for the sharpinfer_b200 native library.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <string>

#include "../../include/sharpinfer_b200.h"

// ---------------------------------------------------------------------------
// Error reporting: every C-ABI call returns an si_status and leaves a
// message retrievable with si_last_error() on the calling thread.
// ---------------------------------------------------------------------------
namespace si {

void set_error(const char* fmt, ...);
void clear_error();

}  // namespace si

#define SI_FAIL(code, ...)        \
  do {                            \
    si::set_error(__VA_ARGS__);   \
    return (code);                \
  } while (0)

#define SI_CUDA(call)                                                              \
  do {                                                                             \
    cudaError_t e_ = (call);                                                       \
    if (e_ != cudaSuccess)                                                         \
      SI_FAIL(SI_ERR_CUDA, "%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), \
              __FILE__, __LINE__);                                                 \
  } while (0)

#define SI_TRY(call)           \
  do {                         \
    int s_ = (call);           \
    if (s_ != SI_OK) return s_; \
  } while (0)

// ---------------------------------------------------------------------------
// Context / weights
// ---------------------------------------------------------------------------

namespace si {
// Tensor parallelism over peer memory.  Every rank owns a communication
// buffer mapped into every other rank (CUDA IPC):
//   [0, 2048)     argmax candidates: [16 batch rows][8 ranks] x two 8-byte
//                 words {value bits, tag}, {index, tag}
//   [2048, ...)   partial sums: [2 kinds][tp source ranks][max_batch][hidden]
//                 8-byte words {f32 bits, tag}
// A producer stores each partial-sum element into slot [kind][own rank] of
// every rank as ONE 8-byte store carrying the value and the step's tag
// (epoch * 2 * n_layers + 2 * layer + kind + 1, never 0).  A consumer polls
// each element it needs until the tag matches -- the 8-byte store is seen
// whole or not at all -- so no fence, counter or flag is needed; it adds the
// tp slots in rank order, so every rank computes the same sum.
constexpr int SI_TP_MAX = 8;
constexpr int SI_TP_ARGMAX = 0, SI_TP_SLOTS = 2048;
struct TpArgs {
  uint8_t* const* peers = nullptr;  // device array [tp] of comm buffer bases
  const unsigned* epoch = nullptr;  // step counter (StepParams::epoch)
  int tp = 1, rank = 0, kind = 0;
  int flag_add = 0;                 // 2 * layer + kind + 1
  int nlayers2 = 0;                 // 2 * n_layers
  int64_t slot_off = 0;             // byte offset of [kind][rank] slots in a comm buffer
  int ld = 0;                       // elements per batch row (hidden)
  __device__ __forceinline__ unsigned tag() const { return *epoch * (unsigned)nlayers2 + (unsigned)flag_add; }
};
// Consumer side of the tensor-parallel sum (k_prep, SI_PREP_RMSNORM_TP).
struct PrepTp {
  const uint8_t* comm = nullptr;    // this rank's comm buffer
  const unsigned* epoch = nullptr;  // step counter
  int* err = nullptr;
  int tp = 1, kind = 0, flag_add = 0, nlayers2 = 0;
  int64_t slots_off = 0;            // byte offset of slots [kind][source 0]
  int64_t src_stride = 0;           // bytes between source ranks' slots
  int ld = 0;                       // elements per batch row
};
// A range of device memory to pull into L2 ahead of the kernel that will read
// it (cp.async.bulk.prefetch.L2): a kernel whose own bytes are already in L2,
// or whose critical path is latency rather than bytes, keeps HBM busy with the
// next kernel's weights.  ptr 16-byte aligned, bytes a multiple of 16, < 4 GB.
struct L2Prefetch {
  const uint8_t* ptr = nullptr;
  uint32_t bytes = 0;
};
// Device scratch of the streaming matvec: partial sums of row tiles split
// between warps ([tiles][slots][64] f32) and per-tile arrival counters
// ([tiles] int, zero between launches).
struct QmvBuffers {
  float* split;
  size_t split_bytes;
  int* count;
  int64_t count_n;
  int* err;
  int sms;
  TpArgs tp;  // used by the SI_EPI_TP epilogue
  L2Prefetch pf;  // weights of a later kernel, pulled into L2 at launch
  int ring_mode;  // batch-1 matvec: when its shared-memory ring is filled (0, 1, 2)
  int q1w;        // batch-1 matvec: warps per CTA (16 or 8)
};
// CTAs (of nw warps) of the streaming matvec for `units` 16x256 units.
inline int64_t qmv_warp_grid(int64_t units, int nw, int sms) {
  int64_t g = units / nw;
  return g < 1 ? 1 : (g > sms ? sms : g);
}
// Scratch a streaming matvec over `tiles` row tiles of `nunit` units needs:
// split floats and counter ints (an upper bound over the ring layouts).
inline void qmv_scratch_need(int64_t tiles, int64_t nunit, int sms, size_t* split_bytes,
                             int64_t* counts, bool wide = true) {
  int64_t worst = 0;
  for (const int nw : {8, 16}) {  // k_qmv_warp: units split over grid x nw warps
    const int64_t units = tiles * nunit, grid = qmv_warp_grid(units, nw, sms);
    const int64_t minr = units / (grid * nw);
    const int64_t maxc = minr > 0 ? (nunit - 1 + minr - 1) / minr + 1 : nunit + 1;
    if (maxc > worst) worst = maxc;
  }
  if (nunit % 2 == 0 && tiles * nunit / 2 >= 16) {  // k_qmv1: unit pairs over grid x 16 warps
    const int64_t P = tiles * nunit / 2, grid = P / 16 < sms ? P / 16 : sms;
    const int64_t minr = P / (grid * 16), npt = nunit / 2;
    const int64_t maxc = (npt - 1 + minr - 1) / minr + 1;
    if (maxc > worst) worst = maxc;
  }
  *split_bytes = (size_t)tiles * worst * 64 * 4;
  // k_qmv_wide: two row-block partials per CTA (a caller without room for
  // them passes wide = false; k_qmv_wide then declines and another kernel runs)
  const size_t tc = (size_t)sms * 2 * 4096 * 4;
  if (wide && *split_bytes < tc) *split_bytes = tc;
  *counts = tiles;
}
}  // namespace si

namespace si {
// One bit per device, set once a one-time per-device step (a kernel's
// shared-memory attribute) has been done there.  Host threads working on
// different GPUs may test and set it concurrently: at worst both do the step.
struct DeviceOnce {
  std::atomic<uint64_t> bits{0};
  bool done(int dev) const { return dev >= 64 || ((bits.load(std::memory_order_acquire) >> dev) & 1u); }
  void mark(int dev) {
    if (dev < 64) bits.fetch_or(1ull << dev, std::memory_order_acq_rel);
  }
};
}  // namespace si

// Grow-only device buffer owned by a context.
struct si_devbuf {
  void* ptr = nullptr;
  size_t bytes = 0;
};

struct si_ctx {
  int device = 0;
  int sm_count = 0;
  size_t l2_bytes = 0;
  cudaStream_t stream = nullptr;
  // Activation staging for the stand-alone quantised matvec: fragment-ordered
  // f16 hi/lo activations, Q4_K sub-block sums and per-vector scales.
  si_devbuf xprep;
  int prep_cols = 0, prep_batch = 0;  // shape of the prepared activations
  int* dev_err = nullptr;             // device error word (SI_DEVERR_* bits)
  si_devbuf qmv_split;                // streaming-matvec split-tile partial sums
  si_devbuf qmv_count;                // and their counters (zero between launches)
  si::QmvBuffers qmv() const {
    return si::QmvBuffers{(float*)qmv_split.ptr, qmv_split.bytes, (int*)qmv_count.ptr,
                          (int64_t)(qmv_count.bytes / 4), dev_err, sm_count, si::TpArgs{}, si::L2Prefetch{}, 0, 16};
  }
  // Host-pointer entry points: device staging and pinned host staging.
  si_devbuf stage[4];
  void* pinned = nullptr;
  size_t pinned_bytes = 0;
};

struct si_weight {
  int qtype = 0;
  int64_t rows = 0, cols = 0;
  int64_t tiles = 0;   // ceil(rows / 16)
  int64_t nblk = 0;    // quant blocks per row
  void* dev = nullptr;
  size_t bytes = 0;
  int device = 0;
  void* f16 = nullptr;  // optional dequantised [rows][cols] f16 copy for prefill (si_qgemm_cache_weight)
};

namespace si {

int ensure(si_devbuf& b, size_t bytes);
int ensure_pinned(si_ctx* c, size_t bytes);
int bind_device(si_ctx* c);
int check_device_errors(si_ctx* c);
int ensure_qmv_scratch(si_ctx* c, const si_weight* w);

// Bytes of one 16-row x one quant block tile in the device layout.
inline int64_t tile_block_bytes(int qt) {
  switch (qt) {
    case SI_Q4_K: return 16 * 144;
    case SI_Q6_K: return 16 * 210;
    case SI_Q8_0: return 16 * 34;
    default: return 0;
  }
}
inline int block_elems(int qt) { return (qt == SI_Q8_0 || qt == SI_Q4_0) ? 32 : 256; }
inline int gguf_block_bytes(int qt) {
  switch (qt) {
    case SI_Q4_K: return 144;
    case SI_Q6_K: return 210;
    case SI_Q8_0: return 34;
    case SI_Q4_0: return 18;
    case SI_Q2_K: return 84;
    case SI_Q3_K: return 110;
    case SI_Q5_K: return 176;
    default: return 0;
  }
}
// Formats kept on the device in their GGUF block layout (rawq.cu): dequant,
// a warp-per-row matvec on f32 activations, and the GEMM's f16 pre-pass.
inline bool raw_layout(int qt) { return qt == SI_Q4_0 || qt == SI_Q2_K || qt == SI_Q3_K || qt == SI_Q5_K; }
int launch_qmv_raw(cudaStream_t s, const si_weight* w, const float* x, float* y, int B);
int launch_dequant_raw(cudaStream_t s, const si_weight* w, float* out);
int launch_dequant_raw_f16(cudaStream_t s, const si_weight* w, __half* out);

// Kernel launchers (defined in the .cu files).
int launch_repack(si_ctx* c, int qt, const uint8_t* gguf, int64_t rows, int64_t cols,
                  int64_t row0, int64_t nrows, void* dst);
int launch_dequant(si_ctx* c, const si_weight* w, float* out);
// Activation preparation modes and matvec epilogues.
enum { SI_PREP_PLAIN = 0, SI_PREP_RMSNORM = 1, SI_PREP_SILU_MUL = 2, SI_PREP_ATTN_MERGE = 3 };
constexpr int SI_ATTN_MAX_SPLITS = 511;
enum { SI_EPI_STORE = 0, SI_EPI_ADD = 1, SI_EPI_TP = 2 };
// mode 4: v = RmsNorm(x + sum of the tp partial-sum slots) * w; the summed
// residual is also written to xout (the next residual buffer)
enum { SI_PREP_RMSNORM_TP = 4 };
constexpr int SI_MAX_K = 49152;  // activation length limit of the prep kernel (smem)
constexpr int SI_MAX_BATCH = 16;

// Prepared activations ("xprep") for K columns and batch B.  Batch b is MMA
// group mg = b/4; a group with Bm batches uses LW = 8*Bm fragment lanes.
// Per group and per 256-column unit (132*LW + 16 bytes): [8 x 32-column
// groups][LW lanes] x 16 B of f16 hi/lo B fragments, LW x 4 B of Q4_K
// sub-block sums, then the 4 inverse activation scales (f32) of the group.
inline int xprep_units(int K) { return (K + 255) / 256; }
inline size_t xprep_bytes(int K, int B) {
  const int nmg = (B + 3) / 4;
  return (size_t)xprep_units(K) * (132 * 8 * B + 16 * nmg);
}

int launch_prep(cudaStream_t s, const float* x, int ldx, const float* x2, const float* norm_w,
                float eps, int mode, int K, int B, float* xout, uint8_t* xprep, bool pdl,
                const PrepTp* tpp = nullptr);
// Batch 5..16 Q4_K / Q6_K matvec over 256-row blocks (k_qmv_wide); -1 when
// the weight, batch or scratch does not suit it.  Switched off by
// SHARPINFER_B200_QMV_WIDE=0 (the one-tile-per-CTA kernel then runs); taken
// from 7168 rows up unless SHARPINFER_B200_QMV_WIDE=2.
int launch_qmv_wide(cudaStream_t s, const si_weight* w, const uint8_t* xprep, int B, float* y, int epi,
                    const QmvBuffers& qb, bool pdl);
bool qmv_wide_enabled();
int launch_qmv(cudaStream_t s, const si_weight* w, const uint8_t* xprep, int B, float* y, int epi,
               const QmvBuffers& qb, bool pdl);
// y (op)= W RmsNorm(x) nw for a single row x (batch 1); xprep is the fallback's
// prepared-activation buffer.
// Tensor parallel, batch 1: y = W RmsNorm(xres + the ranks' partial sums) nw,
// the new residual written to xout, in one batch-1 Q4_K kernel; -1 when that
// kernel does not apply (then k_prep's SI_PREP_RMSNORM_TP and a matvec).
int launch_qmv_rms_tp(cudaStream_t s, const si_weight* w, const float* xres, float* xout, const float* nw, float eps,
                      float* y, const QmvBuffers& qb, const PrepTp& pt, bool pdl);
int launch_qmv_rms(cudaStream_t s, const si_weight* w, const float* x, const float* nw, float eps, float* y,
                   int epi, const QmvBuffers& qb, uint8_t* xprep, bool pdl);
// y (op)= W (SiLU(gate) * up) for one row (batch 1).
int launch_qmv_silu(cudaStream_t s, const si_weight* w, const float* gate, const float* up, float* y, int epi,
                    const QmvBuffers& qb, uint8_t* xprep, bool pdl);
// Prefill GEMM core: y[m] (+)= rs[m] * (xf[m] . W) for f16 rows xf [M][cols]
// scaled per row by rs[m]^-1 (a power of two); accumulate != 0 adds to y.
int launch_qgemm_f16in(si_ctx* c, const si_weight* w, const __half* xf, const float* rs, float* y, int M,
                       int accumulate);
// Prefill attention on 16-bit q, k, v (bf16, or f16 when f16 is set).
int launch_attn_prefill(si_ctx* c, const uint16_t* q, const uint16_t* k, const uint16_t* v, float* o, int batch,
                        int heads, int kv_heads, int seq, int kv, float scale, int causal, int start_pos, bool f16);
int launch_synth_blocks(si_ctx* c, int qt, uint64_t seed, uint64_t tag, int recipe, float sigma,
                        int64_t blk0, int64_t nblocks, uint8_t* dst);
int launch_synth_blocks_2d(si_ctx* c, int qt, uint64_t seed, uint64_t tag, int recipe, float sigma, int64_t grow0,
                           int64_t nrows, int64_t gnblk, int64_t gb0, int64_t nblk, uint8_t* dst);

}  // namespace si

// ---------------------------------------------------------------------------
// Device helpers
// ---------------------------------------------------------------------------
namespace si {

__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t mask, uint32_t orv) {
  uint32_t r;
  // (a & b) | c  -> LUT 0xEA
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(mask), "r"(orv));
  return r;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

__device__ __forceinline__ uint32_t hfma2_u32(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}

__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

__device__ __forceinline__ uint32_t hsub2_u32(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// D = A(16x16 f16, row) * B(16x8 f16, col) + C (f32).  No side effects beyond
// its registers, so the compiler may schedule it freely.
__device__ __forceinline__ void mma16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ uint2 ldg_nc_v2(const void* p) {
  uint2 r;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
               : "=r"(r.x), "=r"(r.y)
               : "l"(p));
  return r;
}

// Programmatic dependent launch controls (no-ops without the launch attribute).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- shared-memory barriers and bulk (TMA engine) copies --------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Wait for phase `parity` of a barrier; gives up after ~200 ms (returns false).
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0; i < (1u << 24); i++) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 255u && globaltimer_ns() - t0 > 200000000ull) return false;
  }
  return false;
}
// After a bounded wait gave up: wait once more, bounded, for each ring stage s
// whose copy may still be in flight (bit s of `pend`; bit s of `par` is the
// phase it completes), so that no bulk copy is still writing shared memory
// when the block moves on.  Worst case ns x 200 ms, not one wait per stage use.
__device__ __forceinline__ void mbar_drain(uint32_t bar0, uint32_t pend, uint32_t par, int ns) {
  for (int s = 0; s < ns; s++)
    if ((pend >> s) & 1u) mbar_wait_bounded(bar0 + 8 * s, (par >> s) & 1u);
}
// Bulk global -> shared copy (16-byte aligned addresses, size a multiple of 16)
// completing `bytes` transactions on the barrier.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}
// The same copy with an L2 evict-first hint: for bytes read exactly once per
// step (weights, KV cache), so that streaming them does not push out lines
// prefetched for the next kernel.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ void bulk_g2s_ef(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar,
                                            uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(bar), "l"(pol)
      : "memory");
}
// This CTA's share of an L2 prefetch: the range split evenly over the grid,
// one prefetch.global.L2 per 128-byte line spread over the CTA's threads.
// Plain load-unit hints, so they never queue ahead of the CTA's own bulk
// copies on the TMA engine.  32-bit arithmetic (a 64-bit division is a long
// subroutine).
__device__ __forceinline__ void l2_prefetch_share(const L2Prefetch& p) {
  if (!p.ptr) return;
  const uint32_t nct = gridDim.x * gridDim.y * gridDim.z;
  const uint32_t cid = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  const uint32_t lines = p.bytes >> 7, per = (lines + nct - 1) / nct;
  const uint32_t a = min(lines, cid * per), b = min(lines, a + per);
  for (uint32_t l = a + threadIdx.x; l < b; l += blockDim.x)
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p.ptr + ((uint64_t)l << 7)));
}
__device__ __forceinline__ uint4 lds_v4(uint32_t a) {
  uint4 r;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(a));
  return r;
}
__device__ __forceinline__ uint2 lds_v2(uint32_t a) {
  uint2 r;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "r"(a));
  return r;
}
__device__ __forceinline__ uint32_t lds_u32(uint32_t a) {
  uint32_t r;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(r) : "r"(a));
  return r;
}

// Device error bits written by kernels whose bounded waits give up.
enum { SI_DEVERR_WAIT_TIMEOUT = 1, SI_DEVERR_PEER_TIMEOUT = 2 };

// ---- tagged 8-byte words between GPUs (peer memory over NVLink) ----
// One 64-bit scalar access (single-copy atomic when 8-byte aligned): value in
// the low word, tag in the high word.
__device__ __forceinline__ void st_tagged(void* p, uint32_t bits, unsigned tag) {
  const uint64_t w = (uint64_t)bits | ((uint64_t)tag << 32);
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ uint2 ld_tagged(const void* p) {
  uint64_t w;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return make_uint2((uint32_t)w, (uint32_t)(w >> 32));
}
// The word at p once its tag is `want` (tags only grow); after ~1 s gives up,
// sets *err and returns what is there.  Once any wait of the step has given up
// (the peer-timeout bit is in *err), later waits return at once: a rank that
// never arrives costs one timeout per step, not one per awaited word.
__device__ __forceinline__ uint32_t wait_tagged(const void* p, unsigned want, int* err) {
  uint2 v = ld_tagged(p);
  if ((int)(v.y - want) >= 0) return v.x;
  const volatile int* verr = err;
  if (*verr & SI_DEVERR_PEER_TIMEOUT) return v.x;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0; i < (1u << 26); i++) {
    v = ld_tagged(p);
    if ((int)(v.y - want) >= 0) return v.x;
    if ((i & 63u) == 63u && ((*verr & SI_DEVERR_PEER_TIMEOUT) || globaltimer_ns() - t0 > 1000000000ull)) break;
  }
  atomicOr(err, SI_DEVERR_PEER_TIMEOUT);
  return v.x;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  return v;
}

}  // namespace si
