// Reading the device weight layout (see quant.cu) back in reference order.
#pragma once
#include "common.cuh"

namespace si {

__device__ __forceinline__ int frag_lane_pos(int k, int* pos) {
  // k in [0,16) -> (t, slot) with slot 0..3 for k = 2t, 2t+1, 2t+8, 2t+9
  int hi = k >> 3, kk = k & 7;
  *pos = 2 * hi + (kk & 1);
  return kk >> 1;
}

__device__ __forceinline__ uint32_t dev_q4k_code(const uint32_t* tbw, int ri, int e) {
  int kt = e >> 4, pos, t = frag_lane_pos(e & 15, &pos);
  int g = ri & 7, upper = ri >> 3, lane = 4 * g + t;
  uint32_t w = tbw[64 + (kt >> 2) * 128 + lane * 4 + (kt & 3)];
  const int sh0[4] = {0, 16, 8, 24}, sh1[4] = {4, 20, 12, 28};
  return (w >> (upper ? sh1[pos] : sh0[pos])) & 0xF;
}

__device__ __forceinline__ uint32_t dev_q6k_code(const uint32_t* tbw, int ri, int e) {
  int kt = e >> 4, pos, t = frag_lane_pos(e & 15, &pos);
  int g = ri & 7, upper = ri >> 3, lane = 4 * g + t;
  int c = kt >> 2, i = kt & 3;
  uint32_t lw = tbw[c * 192 + lane * 4 + i];
  uint32_t hw = tbw[c * 192 + 128 + lane * 2 + (i >> 1)];
  const int sh0[4] = {0, 16, 8, 24}, sh1[4] = {4, 20, 12, 28};
  const int hb0[4] = {4, 20, 12, 28}, hb1[4] = {8, 24, 0, 16};
  uint32_t lo = (lw >> (upper ? sh1[pos] : sh0[pos])) & 0xF;
  uint32_t hi = (hw >> ((upper ? hb1[pos] : hb0[pos]) + 2 * (i & 1))) & 3;
  return lo | (hi << 4);
}

__device__ __forceinline__ int dev_q80_code(const uint32_t* tbw, int ri, int e) {
  int kt = e >> 4, pos, t = frag_lane_pos(e & 15, &pos);
  int g = ri & 7, upper = ri >> 3, lane = 4 * g + t;
  uint32_t w = tbw[lane * 4 + kt * 2 + upper];
  return (int)(int8_t)((w >> (8 * pos)) & 0xFF);
}

__device__ __forceinline__ float h2f(uint32_t bits16) {
  return __half2float(__ushort_as_half((unsigned short)bits16));
}

// Elements of quant block b of row r, in reference order and with the
// reference's rounding (no FMA contraction): DequantQ4_K
// (Quantization.cs:273-314), DequantQ6_K (:362-391), DequantQ8_0 (:106-114).
__device__ __forceinline__ void dequant_block(int qt, const uint8_t* __restrict__ W, int64_t nblk,
                                              int64_t r, int64_t b, float* __restrict__ o) {
  const int64_t T = r >> 4;
  const int ri = (int)(r & 15);
  if (qt == SI_Q4_K) {
    const uint32_t* tbw = (const uint32_t*)(W + (T * nblk + b) * 2304);
    const uint8_t* hdr = (const uint8_t*)(tbw + 4 * ri);
    const float d = h2f(hdr[0] | (hdr[1] << 8)), dmin = h2f(hdr[2] | (hdr[3] << 8));
    const uint8_t* q = hdr + 4;
    for (int j = 0; j < 8; j++) {  // GetScaleMinK4 (Quantization.cs:302-314)
      uint32_t sc, mn;
      if (j < 4) {
        sc = q[j] & 63;
        mn = q[j + 4] & 63;
      } else {
        sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        mn = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
      }
      const float d1 = __fmul_rn(d, (float)sc), m1f = __fmul_rn(dmin, (float)mn);
      for (int l = 0; l < 32; l++) {
        const int e = 32 * j + l;
        o[e] = __fsub_rn(__fmul_rn(d1, (float)dev_q4k_code(tbw, ri, e)), m1f);
      }
    }
  } else if (qt == SI_Q6_K) {
    const uint32_t* tbw = (const uint32_t*)(W + (T * nblk + b) * 3360);
    const int8_t* scales = (const int8_t*)(tbw + 768) + 16 * ri;
    const uint32_t dw = tbw[832 + (ri & 7)];
    const float d = h2f((ri >> 3) ? (dw >> 16) : (dw & 0xFFFF));
    for (int e = 0; e < 256; e++) {
      const float ds = __fmul_rn(d, (float)scales[e >> 4]);
      o[e] = __fmul_rn(ds, (float)((int)dev_q6k_code(tbw, ri, e) - 32));
    }
  } else {
    const uint32_t* tbw = (const uint32_t*)(W + (T * nblk + b) * 544);
    const uint32_t dw = tbw[128 + (ri & 7)];
    const float d = h2f((ri >> 3) ? (dw >> 16) : (dw & 0xFFFF));
    for (int e = 0; e < 32; e++) o[e] = __fmul_rn((float)dev_q80_code(tbw, ri, e), d);
  }
}

// Element `col` of row r of a device-layout weight (reference rounding).
__device__ __forceinline__ float dev_weight_elem(int qt, const uint8_t* __restrict__ W, int64_t nblk,
                                             int64_t r, int col) {
  const int64_t T = r >> 4;
  const int ri = (int)(r & 15);
  if (qt == SI_Q4_K) {
    const int64_t b = col >> 8;
    const int e = col & 255, j = e >> 5;
    const uint32_t* tbw = (const uint32_t*)(W + (T * nblk + b) * 2304);
    const uint8_t* hdr = (const uint8_t*)(tbw + 4 * ri);
    const float d = h2f(hdr[0] | (hdr[1] << 8)), dmin = h2f(hdr[2] | (hdr[3] << 8));
    const uint8_t* q = hdr + 4;
    uint32_t sc, mn;
    if (j < 4) {
      sc = q[j] & 63;
      mn = q[j + 4] & 63;
    } else {
      sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
      mn = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
    const float d1 = __fmul_rn(d, (float)sc), m1f = __fmul_rn(dmin, (float)mn);
    return __fsub_rn(__fmul_rn(d1, (float)dev_q4k_code(tbw, ri, e)), m1f);
  } else if (qt == SI_Q6_K) {
    const int64_t b = col >> 8;
    const int e = col & 255;
    const uint32_t* tbw = (const uint32_t*)(W + (T * nblk + b) * 3360);
    const int8_t* scales = (const int8_t*)(tbw + 768) + 16 * ri;
    const uint32_t dw = tbw[832 + (ri & 7)];
    const float d = h2f((ri >> 3) ? (dw >> 16) : (dw & 0xFFFF));
    const float ds = __fmul_rn(d, (float)scales[e >> 4]);
    return __fmul_rn(ds, (float)((int)dev_q6k_code(tbw, ri, e) - 32));
  } else {
    const int64_t b = col >> 5;
    const int e = col & 31;
    const uint32_t* tbw = (const uint32_t*)(W + (T * nblk + b) * 544);
    const uint32_t dw = tbw[128 + (ri & 7)];
    const float d = h2f((ri >> 3) ? (dw >> 16) : (dw & 0xFFFF));
    return __fmul_rn((float)dev_q80_code(tbw, ri, e), d);
  }
}

}  // namespace si
