// GGUF K-quant blocks <-> the device layout, bit-exact dequantisation and the
// on-device synthetic block generator.
//
// Device layout.  Rows are grouped in tiles of 16 (zero-padded at the end).
// Tile T and quant block b form one "tile-block" of 16 x (GGUF block bytes)
// bytes, stored at ((T * nblk) + b) * tile_block_bytes, so a row tile streams
// its blocks contiguously.  Inside a tile-block the quants are stored in the
// order in which mma.m16n8k16 wants its A fragment: lane (g = lane/4,
// t = lane%4) holds rows g and g+8 at k = 2t, 2t+1, 2t+8, 2t+9 of every
// 16-element k-tile.  One 32-bit word carries those 8 values:
//   bits 0-3 : row g,   k=2t      bits 16-19: row g,   k=2t+1
//   bits 4-7 : row g+8, k=2t      bits 20-23: row g+8, k=2t+1
//   bits 8-11: row g,   k=2t+8    bits 24-27: row g,   k=2t+9
//   bits12-15: row g+8, k=2t+8    bits 28-31: row g+8, k=2t+9
// so `(w & 0x000F000F) | 0x64006400` is the f16 pair (1024+q0, 1024+q1) and
// `(w & 0x00F000F0) | 0x64006400` the pair (1024+16 q2, 1024+16 q3).
//
//  Q4_K tile-block (2304 B): [16 rows x 16 B GGUF header (d, dmin, scales)]
//                            [4 chunks x 32 lanes x 4 words]  (chunk = 4 k-tiles)
//  Q6_K tile-block (3360 B): [4 chunks x (32 lanes x 4 low-nibble words +
//                                        32 lanes x 2 high-bit words)]
//                            [16 rows x 16 int8 scales][8 x (d_g, d_g+8) f16]
//  Q8_0 tile-block (544 B) : [32 lanes x 4 words: (row g, kt0), (row g+8, kt0),
//                                                  (row g, kt1), (row g+8, kt1)]
//                            [8 x (d_g, d_g+8) f16]
// Q6_K high bits of k-tile 2j (k-tile 2j+1 is the same pattern shifted left
// by 2): row g k=2t -> bits 4-5, k=2t+1 -> 20-21, k=2t+8 -> 12-13,
// k=2t+9 -> 28-29; row g+8 k=2t -> 8-9, k=2t+1 -> 24-25, k=2t+8 -> 0-1,
// k=2t+9 -> 16-17.
//
// GGUF decoding follows src/SharpInfer.Core/Tensors/Quantization.cs:
// Q4_K :273-314, Q6_K :362-391, Q8_0 :106-114.
#include <stdio.h>

#include "common.cuh"
#include "quantfmt.cuh"
#include "synth.h"

namespace si {
namespace {

// Quant code of (row, element e) of one GGUF block.
__device__ __forceinline__ uint32_t q4k_code(const uint8_t* blk, int e) {
  int p = e >> 6, l = e & 63;
  uint8_t byte = blk[16 + 32 * p + (l & 31)];
  return l < 32 ? (byte & 0xF) : (byte >> 4);
}

__device__ __forceinline__ uint32_t q6k_code(const uint8_t* blk, int e) {
  int n = e >> 7, w = e & 127, k = w >> 5, l = w & 31;
  const uint8_t* ql = blk;
  const uint8_t* qh = blk + 128;
  uint32_t lo = (k & 1) ? ql[64 * n + l + 32] : ql[64 * n + l];
  lo = (k & 2) ? (lo >> 4) : (lo & 0xF);
  uint32_t hi = (qh[32 * n + l] >> (2 * k)) & 3;
  return lo | (hi << 4);
}

__device__ __forceinline__ uint32_t q80_code(const uint8_t* blk, int e) { return blk[2 + e]; }

// Pointer to GGUF block (row r, block b) in a staging buffer that holds rows
// [row0, row0 + nrows); NULL for padding rows.
__device__ __forceinline__ const uint8_t* src_block(const uint8_t* src, int64_t r, int64_t b,
                                                    int64_t row0, int64_t rows, int64_t nblk,
                                                    int bb) {
  if (r >= rows) return nullptr;
  return src + ((r - row0) * nblk + b) * bb;
}

// One thread per 32-bit word of the device layout.
__global__ void k_repack(int qt, const uint8_t* __restrict__ src, int64_t row0, int64_t rows,
                         int64_t nblk, int64_t tile0, int64_t ntiles, uint32_t* __restrict__ dst) {
  const int bb = qt == SI_Q4_K ? 144 : (qt == SI_Q6_K ? 210 : 34);
  const int wpt = (16 * bb) / 4;  // words per tile-block
  int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t total = ntiles * nblk * wpt;
  if (idx >= total) return;
  int wi = (int)(idx % wpt);
  int64_t tb = idx / wpt;
  int64_t b = tb % nblk;
  int64_t T = tile0 + tb / nblk;
  uint32_t out = 0;
  if (qt == SI_Q4_K) {
    if (wi < 64) {  // verbatim header word
      int ri = wi >> 2, j = wi & 3;
      const uint8_t* s = src_block(src, 16 * T + ri, b, row0, rows, nblk, bb);
      if (s) out = s[4 * j] | (s[4 * j + 1] << 8) | (s[4 * j + 2] << 16) | ((uint32_t)s[4 * j + 3] << 24);
    } else {
      int q = wi - 64, c = q >> 7, lane = (q & 127) >> 2, i = q & 3;
      int kt = 4 * c + i, g = lane >> 2, t = lane & 3;
      const uint8_t* s0 = src_block(src, 16 * T + g, b, row0, rows, nblk, bb);
      const uint8_t* s1 = src_block(src, 16 * T + g + 8, b, row0, rows, nblk, bb);
      int e0 = 16 * kt + 2 * t;
      const int ks[4] = {e0, e0 + 1, e0 + 8, e0 + 9};
      const int sh0[4] = {0, 16, 8, 24};  // row g
      const int sh1[4] = {4, 20, 12, 28};  // row g+8
      for (int j = 0; j < 4; j++) {
        if (s0) out |= q4k_code(s0, ks[j]) << sh0[j];
        if (s1) out |= q4k_code(s1, ks[j]) << sh1[j];
      }
    }
  } else if (qt == SI_Q6_K) {
    if (wi < 768) {
      int c = wi / 192, r = wi % 192;
      const int sh0[4] = {0, 16, 8, 24}, sh1[4] = {4, 20, 12, 28};
      const int hb0[4] = {4, 20, 12, 28}, hb1[4] = {8, 24, 0, 16};
      if (r < 128) {  // low nibbles of k-tile 4c + i
        int lane = r >> 2, i = r & 3, kt = 4 * c + i, g = lane >> 2, t = lane & 3;
        const uint8_t* s0 = src_block(src, 16 * T + g, b, row0, rows, nblk, bb);
        const uint8_t* s1 = src_block(src, 16 * T + g + 8, b, row0, rows, nblk, bb);
        int e0 = 16 * kt + 2 * t;
        const int ks[4] = {e0, e0 + 1, e0 + 8, e0 + 9};
        for (int j = 0; j < 4; j++) {
          if (s0) out |= (q6k_code(s0, ks[j]) & 0xF) << sh0[j];
          if (s1) out |= (q6k_code(s1, ks[j]) & 0xF) << sh1[j];
        }
      } else {  // high 2-bit fields of k-tiles 4c + 2j and 4c + 2j + 1
        int r2 = r - 128, lane = r2 >> 1, jj = r2 & 1, g = lane >> 2, t = lane & 3;
        const uint8_t* s0 = src_block(src, 16 * T + g, b, row0, rows, nblk, bb);
        const uint8_t* s1 = src_block(src, 16 * T + g + 8, b, row0, rows, nblk, bb);
        for (int half = 0; half < 2; half++) {
          int kt = 4 * c + 2 * jj + half;
          int e0 = 16 * kt + 2 * t;
          const int ks[4] = {e0, e0 + 1, e0 + 8, e0 + 9};
          for (int j = 0; j < 4; j++) {
            if (s0) out |= (q6k_code(s0, ks[j]) >> 4) << (hb0[j] + 2 * half);
            if (s1) out |= (q6k_code(s1, ks[j]) >> 4) << (hb1[j] + 2 * half);
          }
        }
      }
    } else if (wi < 832) {  // int8 scales, 16 per row
      int ri = (wi - 768) >> 2, j = (wi - 768) & 3;
      const uint8_t* s = src_block(src, 16 * T + ri, b, row0, rows, nblk, bb);
      if (s)
        out = s[192 + 4 * j] | (s[193 + 4 * j] << 8) | (s[194 + 4 * j] << 16) |
              ((uint32_t)s[195 + 4 * j] << 24);
    } else {  // (d_g, d_g+8)
      int g = wi - 832;
      const uint8_t* s0 = src_block(src, 16 * T + g, b, row0, rows, nblk, bb);
      const uint8_t* s1 = src_block(src, 16 * T + g + 8, b, row0, rows, nblk, bb);
      if (s0) out |= s0[208] | (s0[209] << 8);
      if (s1) out |= ((uint32_t)s1[208] << 16) | ((uint32_t)s1[209] << 24);
    }
  } else {  // Q8_0
    if (wi < 128) {
      int lane = wi >> 2, j = wi & 3, kt = j >> 1, which = j & 1, g = lane >> 2, t = lane & 3;
      const uint8_t* s = src_block(src, 16 * T + g + 8 * which, b, row0, rows, nblk, bb);
      int e0 = 16 * kt + 2 * t;
      if (s)
        out = q80_code(s, e0) | (q80_code(s, e0 + 1) << 8) | (q80_code(s, e0 + 8) << 16) |
              (q80_code(s, e0 + 9) << 24);
    } else {
      int g = wi - 128;
      const uint8_t* s0 = src_block(src, 16 * T + g, b, row0, rows, nblk, bb);
      const uint8_t* s1 = src_block(src, 16 * T + g + 8, b, row0, rows, nblk, bb);
      if (s0) out |= s0[0] | (s0[1] << 8);
      if (s1) out |= ((uint32_t)s1[0] << 16) | ((uint32_t)s1[1] << 24);
    }
  }
  dst[(T * nblk + b) * wpt + wi] = out;
}

// One thread per (row, quant block): writes the block's elements in
// reference order with the reference's rounding (no FMA contraction).
__global__ void k_dequant(int qt, const uint8_t* __restrict__ W, int64_t rows, int64_t nblk,
                          float* __restrict__ out) {
  int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= rows * nblk) return;
  const int64_t r = idx / nblk, b = idx % nblk;
  const int be = qt == SI_Q8_0 ? 32 : 256;
  dequant_block(qt, W, nblk, r, b, out + r * nblk * be + b * be);
}

// Blocks blk0 + i (i < nblocks) of a tensor, or -- when nblk > 0 -- the
// blocks of rows grow0 .. grow0 + nblocks / nblk, columns gb0 .. gb0 + nblk of
// a tensor with gnblk blocks per row (a slice of every row), row-major.
__global__ void k_synth_blocks(int qt, uint64_t key, int recipe, float sigma, int64_t blk0,
                               int64_t nblocks, uint8_t* __restrict__ dst, int64_t gnblk, int64_t gb0,
                               int64_t nblk) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nblocks) return;
  uint64_t gb = nblk > 0 ? (uint64_t)((blk0 + i / nblk) * gnblk + gb0 + i % nblk) : (uint64_t)(blk0 + i);
  uint8_t buf[210];
  int bb;
  if (qt == SI_Q4_K) {
    si_synth_q4k_block(key, gb, sigma, recipe, buf);
    bb = 144;
  } else if (qt == SI_Q6_K) {
    si_synth_q6k_block(key, gb, sigma, buf);
    bb = 210;
  } else {
    si_synth_q80_block(key, gb, sigma, buf);
    bb = 34;
  }
  uint8_t* o = dst + i * bb;
  for (int k = 0; k < bb; k++) o[k] = buf[k];
}

}  // namespace

int launch_repack(si_ctx* c, int qt, const uint8_t* gguf, int64_t rows, int64_t cols,
                  int64_t row0, int64_t nrows, void* dst) {
  int64_t nblk = cols / block_elems(qt);
  int64_t tile0 = row0 / 16;
  int64_t ntiles = (nrows + 15) / 16;
  int64_t words = ntiles * nblk * (tile_block_bytes(qt) / 4);
  if (words == 0) return SI_OK;
  int threads = 256;
  int64_t blocks = (words + threads - 1) / threads;
  k_repack<<<(unsigned)blocks, threads, 0, c->stream>>>(qt, gguf, row0, rows, nblk, tile0, ntiles,
                                                        (uint32_t*)dst);
  SI_CUDA(cudaGetLastError());
  return SI_OK;
}

int launch_dequant(si_ctx* c, const si_weight* w, float* out) {
  int64_t n = w->rows * w->nblk;
  if (n == 0) return SI_OK;
  int threads = 128;
  k_dequant<<<(unsigned)((n + threads - 1) / threads), threads, 0, c->stream>>>(
      w->qtype, (const uint8_t*)w->dev, w->rows, w->nblk, out);
  SI_CUDA(cudaGetLastError());
  return SI_OK;
}

int launch_synth_blocks(si_ctx* c, int qt, uint64_t seed, uint64_t tag, int recipe, float sigma,
                        int64_t blk0, int64_t nblocks, uint8_t* dst) {
  if (nblocks == 0) return SI_OK;
  int threads = 128;
  k_synth_blocks<<<(unsigned)((nblocks + threads - 1) / threads), threads, 0, c->stream>>>(
      qt, si_key(seed, tag), recipe, sigma, blk0, nblocks, dst, 0, 0, 0);
  SI_CUDA(cudaGetLastError());
  return SI_OK;
}

int launch_synth_blocks_2d(si_ctx* c, int qt, uint64_t seed, uint64_t tag, int recipe, float sigma, int64_t grow0,
                           int64_t nrows, int64_t gnblk, int64_t gb0, int64_t nblk, uint8_t* dst) {
  const int64_t nblocks = nrows * nblk;
  if (nblocks == 0) return SI_OK;
  int threads = 128;
  k_synth_blocks<<<(unsigned)((nblocks + threads - 1) / threads), threads, 0, c->stream>>>(
      qt, si_key(seed, tag), recipe, sigma, grow0, nblocks, dst, gnblk, gb0, nblk);
  SI_CUDA(cudaGetLastError());
  return SI_OK;
}

}  // namespace si
