// Seeded synthetic GGUF blocks, activations and KV entries.
//
// Every value is a pure function of (seed, tensor tag, element index) built
// from integer hashing, one int->float conversion and one IEEE multiply, so
// the same bytes come out of the host routine and the device kernel.  The
// device generator fills multi-GB weight sets in place (no PCIe traffic);
// the host generator feeds the CPU oracle the identical bytes.
//
// Distributions (weights of a fresh model, not trained values):
//   normal(z)  : Irwin-Hall sum of four 16-bit uniforms, scaled to unit
//                variance (bounded by +-3.46 sigma).
//   Q4_K       : d, dmin = f16(|z| * sigma); 6-bit sc, m; nibbles uniform.
//   Q6_K       : d = f16(|z| * sigma); int8 scales uniform in [-32, 32];
//                6-bit quants uniform.
//   Q8_0       : d = f16(|z| * sigma); int8 quants uniform.
// Block layouts are the GGML ones decoded by
// src/SharpInfer.Core/Tensors/Quantization.cs (Q4_K :273-314, Q6_K :362-391,
// Q8_0 :106-114).
#pragma once
#include <math.h>
#include <stdint.h>

#if defined(__CUDACC__)
#define SI_HD __host__ __device__ __forceinline__
#else
#define SI_HD static inline
#endif

// Separately rounded multiply and add (no FMA contraction on either side).
#if defined(__CUDA_ARCH__)
#define SI_FMUL(a, b) __fmul_rn((a), (b))
#define SI_FADD(a, b) __fadd_rn((a), (b))
#else
#define SI_FMUL(a, b) ((a) * (b))
#define SI_FADD(a, b) ((a) + (b))
#endif

#define SI_GOLDEN 0x9E3779B97F4A7C15ull

SI_HD uint64_t si_mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Stream key for one tensor.
SI_HD uint64_t si_key(uint64_t seed, uint64_t tag) {
  return si_mix64(seed ^ si_mix64(tag + SI_GOLDEN));
}

// 64 random bits for draw `idx` of stream `key`.
SI_HD uint64_t si_bits(uint64_t key, uint64_t idx) {
  return si_mix64(key + (idx + 1) * SI_GOLDEN);
}

// Approximately standard-normal draw from 64 bits.
SI_HD float si_normal(uint64_t r) {
  int32_t s = (int32_t)(r & 0xFFFF) + (int32_t)((r >> 16) & 0xFFFF) +
              (int32_t)((r >> 32) & 0xFFFF) + (int32_t)(r >> 48) - 131070;
  return SI_FMUL((float)s, 2.6428903e-05f);  // 1 / sqrt(4 * (65536^2 - 1) / 12)
}

// IEEE binary32 -> binary16, round to nearest even (integer code, so host and
// device agree bit for bit).
SI_HD uint16_t si_f32_to_f16(float f) {
  union { float f; uint32_t u; } v;
  v.f = f;
  uint32_t x = v.u;
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t ax = x & 0x7FFFFFFFu;
  if (ax >= 0x7F800000u) {  // inf / nan
    return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0u));
  }
  if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);  // rounds to inf
  if (ax < 0x38800000u) {  // result is subnormal or zero
    if (ax < 0x33000000u) return (uint16_t)sign;  // < 2^-25 -> 0
    uint32_t e = ax >> 23;
    uint32_t m = (ax & 0x7FFFFFu) | 0x800000u;
    uint32_t shift = 126u - e;  // value / 2^-24 = mantissa >> (126 - e)
    uint32_t q = m >> shift;
    uint32_t rem = m & ((1u << shift) - 1u);
    uint32_t half = 1u << (shift - 1u);
    if (rem > half || (rem == half && (q & 1u))) q++;
    return (uint16_t)(sign | q);
  }
  uint32_t e = (ax >> 23) - 112u;
  uint32_t m = ax & 0x7FFFFFu;
  uint32_t q = (e << 10) | (m >> 13);
  uint32_t rem = m & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
  return (uint16_t)(sign | q);
}

// IEEE binary16 -> binary32 (exact).
SI_HD float si_f16_to_f32(uint16_t h) {
  uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
  uint32_t e = ((uint32_t)h >> 10) & 0x1Fu;
  uint32_t m = (uint32_t)h & 0x3FFu;
  uint32_t u;
  if (e == 0) {
    if (m == 0) {
      u = sign;
    } else {  // subnormal: normalise
      e = 113;
      while ((m & 0x400u) == 0) { m <<= 1; e--; }
      m &= 0x3FFu;
      u = sign | (e << 23) | (m << 13);
    }
  } else if (e == 31) {
    u = sign | 0x7F800000u | (m << 13);
  } else {
    u = sign | ((e + 112u) << 23) | (m << 13);
  }
  union { uint32_t u; float f; } v;
  v.u = u;
  return v.f;
}

// Recipes (`recipe` argument).  `sigma` scales |z| for the block scale d (and
// dmin).  0: the distributions listed in the header comment; 1: zero-mean
// Q4_K weights for model tensors: sc in 1..8, m = round(7.5 sc), dmin = d.
#define SI_RECIPE_MODEL 1

// One Q4_K block (144 bytes): [f16 d][f16 dmin][12 packed scales][128 qs].
SI_HD void si_synth_q4k_block(uint64_t key, uint64_t blk, float sigma, int recipe,
                              uint8_t* out) {
  uint64_t base = blk * 20u;
  uint64_t r0 = si_bits(key, base + 0);
  uint64_t r1 = si_bits(key, base + 1);
  uint64_t r2 = si_bits(key, base + 2);
  uint16_t d = si_f32_to_f16(SI_FMUL(fabsf(si_normal(r0)), sigma));
  uint16_t dmin;
  uint8_t sc[8], m[8];
  if (recipe == SI_RECIPE_MODEL) {
    dmin = d;
    for (int j = 0; j < 8; j++) {
      uint32_t s = 1u + (uint32_t)((r2 >> (3 * j)) & 7u);
      sc[j] = (uint8_t)s;
      m[j] = (uint8_t)((15u * s + 1u) / 2u);
    }
  } else {
    dmin = si_f32_to_f16(SI_FMUL(fabsf(si_normal(r1)), sigma));
    uint64_t r3 = si_bits(key, base + 3);
    for (int j = 0; j < 8; j++) {
      sc[j] = (uint8_t)((r2 >> (6 * j)) & 63u);
      m[j] = (uint8_t)((r3 >> (6 * j)) & 63u);
    }
  }
  out[0] = (uint8_t)(d & 0xFF);
  out[1] = (uint8_t)(d >> 8);
  out[2] = (uint8_t)(dmin & 0xFF);
  out[3] = (uint8_t)(dmin >> 8);
  // Inverse of GetScaleMinK4 (Quantization.cs:302-314).
  for (int i = 0; i < 4; i++) {
    out[4 + i] = (uint8_t)(sc[i] | ((sc[i + 4] >> 4) << 6));
    out[8 + i] = (uint8_t)(m[i] | ((m[i + 4] >> 4) << 6));
    out[12 + i] = (uint8_t)((sc[i + 4] & 0xF) | ((m[i + 4] & 0xF) << 4));
  }
  for (int w = 0; w < 16; w++) {
    uint64_t r = si_bits(key, base + 4 + w);
    for (int b = 0; b < 8; b++) out[16 + 8 * w + b] = (uint8_t)(r >> (8 * b));
  }
}

// One Q6_K block (210 bytes): [128 ql][64 qh][16 int8 scales][f16 d].
SI_HD void si_synth_q6k_block(uint64_t key, uint64_t blk, float sigma, uint8_t* out) {
  uint64_t base = blk * 28u;
  uint16_t d = si_f32_to_f16(SI_FMUL(fabsf(si_normal(si_bits(key, base))), sigma));
  for (int w = 0; w < 24; w++) {  // 192 bytes of ql + qh: all 6-bit codes uniform
    uint64_t r = si_bits(key, base + 1 + w);
    for (int b = 0; b < 8; b++) out[8 * w + b] = (uint8_t)(r >> (8 * b));
  }
  for (int j = 0; j < 16; j++) {
    uint64_t r = si_bits(key, base + 25 + (j >> 3));
    uint32_t v = (uint32_t)((r >> (8 * (j & 7))) & 0xFFu);
    int s = (int)(v % 65u) - 32;  // [-32, 32]
    out[192 + j] = (uint8_t)(int8_t)s;
  }
  out[208] = (uint8_t)(d & 0xFF);
  out[209] = (uint8_t)(d >> 8);
}

// One Q8_0 block (34 bytes): [f16 d][32 int8].
SI_HD void si_synth_q80_block(uint64_t key, uint64_t blk, float sigma, uint8_t* out) {
  uint64_t base = blk * 5u;
  uint16_t d = si_f32_to_f16(SI_FMUL(fabsf(si_normal(si_bits(key, base))), sigma));
  out[0] = (uint8_t)(d & 0xFF);
  out[1] = (uint8_t)(d >> 8);
  for (int w = 0; w < 4; w++) {
    uint64_t r = si_bits(key, base + 1 + w);
    for (int b = 0; b < 8; b++) out[2 + 8 * w + b] = (uint8_t)(r >> (8 * b));
  }
}

// f32 element i of a normal(mean, sigma) vector.
SI_HD float si_synth_f32(uint64_t key, uint64_t i, float mean, float sigma) {
  return SI_FADD(mean, SI_FMUL(si_normal(si_bits(key, i)), sigma));
}

// f16 element i of a normal(0, sigma) vector (KV cache fill).
SI_HD uint16_t si_synth_f16(uint64_t key, uint64_t i, float sigma) {
  return si_f32_to_f16(SI_FMUL(si_normal(si_bits(key, i)), sigma));
}
