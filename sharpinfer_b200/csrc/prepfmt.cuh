// The prepared-activation format shared by every producer of matvec inputs
// (k_prep, the fused RmsNorm of the batch-1 Q4_K matvec, the attention split
// merge): per 256-column unit and MMA group of up to 4 batch rows, the values
// scaled by 2^e (max |v 2^e| in [2^13, 2^14)), split into f16 hi + lo
// fragments in mma.m16n8k16 B-operand order, the Q4_K sub-block sums, and the
// inverse scales.
#pragma once
#include "common.cuh"

namespace si {

constexpr int XUNIT_LANES_FULL = 32;

// Split v into f16 hi + lo; part 0 -> hi, 1 -> lo.
__device__ __forceinline__ __half split_part(float v, int part) {
  __half hi = __float2half_rn(v);
  if (part == 0) return hi;
  return __float2half_rn(v - __half2float(hi));
}

__device__ __forceinline__ uint32_t pack2(__half a, __half b) {
  return (uint32_t)__half_as_ushort(a) | ((uint32_t)__half_as_ushort(b) << 16);
}

// Sum of the 32 values of Q4_K sub-block lane / 4 of a 256-value unit in
// shared memory (16-byte aligned), returned in the four lanes 4j .. 4j + 3 of
// sub-block j: each lane adds 8 consecutive values, then the four partial
// sums are combined.  The order is fixed, so every producer gets the same sums.
__device__ __forceinline__ float subblock_sum(const float* sv, int lane) {
  const float4 a = *(const float4*)(sv + 8 * lane), b = *(const float4*)(sv + 8 * lane + 4);
  float p = ((a.x + a.y) + (a.z + a.w)) + ((b.x + b.y) + (b.z + b.w));
  p += __shfl_xor_sync(0xFFFFFFFFu, p, 1);
  return p + __shfl_xor_sync(0xFFFFFFFFu, p, 2);
}

// Byte offset of MMA group mg, unit u in the prepared-activation buffer.
// A unit of a group with LW lanes is 132*LW + 16 bytes: fragments, Q4_K
// sub-block sums, then the 4 inverse activation scales of the group.
__device__ __forceinline__ int xunit_bytes(int LW) { return 132 * LW + 16; }
__device__ __forceinline__ int64_t xprep_off(int mg, int nunit, int u, int LW) {
  return (int64_t)mg * nunit * xunit_bytes(XUNIT_LANES_FULL) + (int64_t)u * xunit_bytes(LW);
}

// Power-of-two exponent e of a unit: max |v 2^e| in [2^13, 2^14).  E is
// read from the exponent bits (amax < 2^E for a normal amax; a subnormal one
// gives E = -126 and e is clamped either way).
__device__ __forceinline__ int unit_exponent(float amax) {
  int e = 0;
  if (amax > 0.f && amax <= 3.0e38f) {
    const int E = (int)((__float_as_uint(amax) >> 23) & 0xFFu) - 126;
    e = 14 - E;
    e = e < -100 ? -100 : (e > 100 ? 100 : e);
  }
  return e;
}
// 2^e for |e| <= 126, exactly, from the exponent bits.
__device__ __forceinline__ float exp2i(int e) { return __uint_as_float((uint32_t)(127 + e) << 23); }

// One warp packs the 256 values sv (shared memory, 16-byte aligned) of batch
// column cb of an MMA group with LW lanes into `unit`.
__device__ __forceinline__ void pack_unit_warp(const float* sv, uint8_t* unit, int LW, int cb, int lane) {
  float amax = 0.f;
  for (int i = lane; i < 256; i += 32) amax = fmaxf(amax, fabsf(sv[i]));
  amax = warp_max(amax);
  const int e = unit_exponent(amax);
  const float sc = exp2i(e);
#pragma unroll
  for (int r = 0; r < 2; r++) {  // fragments: 8 groups x (hi, lo) x 4 lanes
    const int task = lane + 32 * r, jj = task >> 3, part = (task >> 2) & 1, t = task & 3;
    uint32_t w[4];
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const int base = 32 * jj + 16 * h + 2 * t;
      const float v0 = sv[base] * sc, v1 = sv[base + 1] * sc, v2 = sv[base + 8] * sc, v3 = sv[base + 9] * sc;
      w[2 * h] = pack2(split_part(v0, part), split_part(v1, part));
      w[2 * h + 1] = pack2(split_part(v2, part), split_part(v3, part));
    }
    *(uint4*)(unit + (jj * LW + 8 * cb + 4 * part + t) * 16) = make_uint4(w[0], w[1], w[2], w[3]);
  }
  // Q4_K sub-block sums (X_{2t}, X_{2t+1}) * 2^-5, then the inverse scale
  const float S = subblock_sum(sv, lane);
  const int part = (lane >> 2) & 1, t = lane & 3;
  const float X0 = __shfl_sync(0xFFFFFFFFu, S, 8 * t), X1 = __shfl_sync(0xFFFFFFFFu, S, 8 * t + 4);
  const float s5 = sc * 0.03125f;
  if (lane < 8)
    *(uint32_t*)(unit + 8 * LW * 16 + (8 * cb + 4 * part + t) * 4) =
        pack2(split_part(X0 * s5, part), split_part(X1 * s5, part));
  else if (lane == 8)
    *(float*)(unit + 132 * LW + 4 * cb) = exp2i(-e);
}

}  // namespace si
