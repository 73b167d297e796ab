// Shared definitions for the sharpinfer_b200 native library.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

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
  si_devbuf xfrag, xsfrag, xscale;
  int prep_cols = 0, prep_batch = 0;  // shape of the prepared activations
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
};

namespace si {

int ensure(si_devbuf& b, size_t bytes);
int ensure_pinned(si_ctx* c, size_t bytes);
int bind_device(si_ctx* c);

// Bytes of one 16-row x one quant block tile in the device layout.
inline int64_t tile_block_bytes(int qt) {
  switch (qt) {
    case SI_Q4_K: return 16 * 144;
    case SI_Q6_K: return 16 * 210;
    case SI_Q8_0: return 16 * 34;
    default: return 0;
  }
}
inline int block_elems(int qt) { return qt == SI_Q8_0 ? 32 : 256; }
inline int gguf_block_bytes(int qt) {
  switch (qt) {
    case SI_Q4_K: return 144;
    case SI_Q6_K: return 210;
    case SI_Q8_0: return 34;
    default: return 0;
  }
}

// Kernel launchers (defined in the .cu files).
int launch_repack(si_ctx* c, int qt, const uint8_t* gguf, int64_t rows, int64_t cols,
                  int64_t row0, int64_t nrows, void* dst);
int launch_dequant(si_ctx* c, const si_weight* w, float* out);
// Activation preparation modes and matvec epilogues.
enum { SI_PREP_PLAIN = 0, SI_PREP_RMSNORM = 1, SI_PREP_SILU_MUL = 2 };
enum { SI_EPI_STORE = 0, SI_EPI_ADD = 1 };
constexpr int SI_MAX_K = 49152;  // activation length limit of the prep kernel (smem)
constexpr int SI_MAX_BATCH = 16;

// Sizes of the prepared-activation buffers for K columns and batch B.
inline size_t xfrag_bytes(int K, int B) { return (size_t)((B + 3) / 4) * (K / 32) * 32 * 16; }
inline size_t xsfrag_bytes(int K, int B) { return (size_t)((B + 3) / 4) * (K / 256 + 1) * 32 * 4; }
inline size_t xscale_bytes(int B) { return (size_t)((B + 3) / 4) * 4 * 4; }

int launch_prep(cudaStream_t s, const float* x, const float* x2, const float* norm_w,
                float eps, int mode, int K, int B, float* xout, uint4* xfrag, uint32_t* xsfrag,
                float* xscale, bool pdl);
int launch_qmv(cudaStream_t s, const si_weight* w, const uint4* xfrag, const uint32_t* xsfrag,
               const float* xscale, int B, float* y, int epi, bool pdl);
int launch_synth_blocks(si_ctx* c, int qt, uint64_t seed, uint64_t tag, int recipe, float sigma,
                        int64_t blk0, int64_t nblocks, uint8_t* dst);

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

// D = A(16x16 f16, row) * B(16x8 f16, col) + C (f32).
__device__ __forceinline__ void mma16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
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
