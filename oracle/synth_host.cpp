// Seeded synthetic inputs for the oracle -- TEST INFRASTRUCTURE ONLY.
//
// The oracle and the B200 library must see the same weights, activations and
// KV prefix.  Both build them from one input generator, the host-safe header
// sharpinfer_b200/csrc/synth.h (pure integer hashing, one int->float
// conversion and one IEEE multiply per value).  Compiling it here lets the
// timed CPU baseline and the reference arm of the benchmark run on
// liboracle.so alone, without loading the library under test.  A CPU test
// checks these bytes against the library's si_synth_*_host for the same
// arguments.
#include <stdint.h>

#include "../sharpinfer_b200/csrc/synth.h"

#define OR_API extern "C" __attribute__((visibility("default")))

enum { OR_Q8_0 = 8, OR_Q4_K = 12, OR_Q6_K = 14 };

// rows*cols/blocksize GGUF blocks of type qt into out (row-major), the bytes of
// si_synth_blocks_host(qt, rows, cols, seed, tag, recipe, sigma).
OR_API int or_synth_blocks(int qt, int64_t rows, int64_t cols, uint64_t seed, uint64_t tag, int recipe,
                           float sigma, uint8_t* out) {
  const int be = qt == OR_Q8_0 ? 32 : 256;
  const int bb = qt == OR_Q4_K ? 144 : qt == OR_Q6_K ? 210 : qt == OR_Q8_0 ? 34 : 0;
  if (!bb || !out || rows <= 0 || cols <= 0 || cols % be) return -1;
  const uint64_t key = si_key(seed, tag);
  const int64_t nb = rows * (cols / be);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < nb; i++) {
    if (qt == OR_Q4_K) si_synth_q4k_block(key, (uint64_t)i, sigma, recipe, out + i * bb);
    else if (qt == OR_Q6_K) si_synth_q6k_block(key, (uint64_t)i, sigma, out + i * bb);
    else si_synth_q80_block(key, (uint64_t)i, sigma, out + i * bb);
  }
  return 0;
}

// n values mean + sigma * N(0,1) (si_synth_f32_host).
OR_API void or_synth_f32(int64_t n, uint64_t seed, uint64_t tag, float mean, float sigma, float* out) {
  const uint64_t key = si_key(seed, tag);
  for (int64_t i = 0; i < n; i++) out[i] = si_synth_f32(key, (uint64_t)i, mean, sigma);
}

// n values f16(sigma * N(0,1)) (si_synth_f16_host).
OR_API void or_synth_f16(int64_t n, uint64_t seed, uint64_t tag, float sigma, uint16_t* out) {
  const uint64_t key = si_key(seed, tag);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; i++) out[i] = si_synth_f16(key, (uint64_t)i, sigma);
}
