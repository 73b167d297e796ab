// Q4_K / Q6_K matvec for batch 5..16 (k_qmv_wide).
//
// y[b][r] = sum_c W[r][c] x[b][c], W in the repacked 16-row-tile layout and x
// in the prepared activation format (per 256-column unit and group of 4
// batch rows: f16 hi + lo fragments in mma.m16n8k16 B order, the Q4_K
// sub-block sums, the inverse scales).
//
// Work item = 256 rows (16 tiles) x one 256-column unit; the items, numbered
// row-block-major, are split into one contiguous range per persistent CTA.
// Warp 0 streams each item's 16 weight units and the unit's prepared
// activations into a 3- or 4-stage shared-memory ring, one bulk copy per unit and
// group, issued from parallel lanes (a 4-D tensor copy of the same 16
// strided units moved only about 14 GB/s per SM).
// Warps 1..8 each own two 16-row tiles of the block: the activation
// fragments of a 16-column step are read from shared memory once and serve
// both tiles and every MMA group, so shared-memory reads stay below the
// weight bytes' HBM time; the quants are unpacked in registers into the MMA
// A operand (the nibble masked in place is the f16 subnormal q 2^-24, times
// the 6-bit scale) and the products accumulate in f32.
//
// Measured on B200 (mma.sync m16n8k16 f16 -> f32: 0.48 per clock per SM):
// at batch 13..16 the 4 MMA groups x 17 MMAs per tile-unit make the MMAs,
// not HBM, the limit; at batch 5..8 HBM is.  The same matvec with the
// unpacked weights in tensor memory as the A operand of tcgen05.mma was
// slower at every batch size: reading a 128 x 16 f16 A operand from tensor
// memory costs about 95 cycles per MMA whatever N is, and N is only 2 x batch.
//
// A row block whose units lie in two or more CTAs' ranges is finished by the
// last of them to arrive (per-block counter), adding the others' partial sums
// in CTA order; the result does not depend on timing.
#include "common.cuh"
#include "prepfmt.cuh"
#include "tcgen05.cuh"

#include <algorithm>
#include <cstdlib>

namespace si {
namespace {

constexpr int WD_TILES = 16;  // tiles per row block; warp 0 produces, warps 1 .. 16 / T compute (T tiles each)
constexpr int WD_XG = 132 * 32 + 16;  // prepared activations of one unit, one full group

template <int QT>
struct WideCfg;
template <>
struct WideCfg<SI_Q4_K> {
  static constexpr int TBB = 2304;  // bytes of a tile unit
};
template <>
struct WideCfg<SI_Q6_K> {
  static constexpr int TBB = 3360;
};
template <int QT>
struct WideSmem {
  static constexpr int TBB = WideCfg<QT>::TBB;
  static constexpr int NS = QT == SI_Q4_K ? 4 : 3;                  // ring stages
  static constexpr int WB = WD_TILES * TBB;                         // weights of one item
  static constexpr int XOFF = (WB + 1023) / 1024 * 1024;            // activations, 1024-aligned
  static constexpr int SB = (XOFF + 4 * WD_XG + 1023) / 1024 * 1024;  // ring stage
  static constexpr int ZERO = NS * SB;                           // zero region (fragments of absent lanes)
  static constexpr int BAR = ZERO + 1024;                           // full[NS] empty[NS]
  static constexpr int MISC = BAR + 16 * NS;                     // last-arriver flag
  static constexpr int SMEM = MISC + 16 + 1024;                     // + alignment slack
  static_assert(SMEM <= 227 * 1024, "shared memory");
};

__device__ __forceinline__ float wd_h2f_lo(uint32_t w) {
  return __half2float(__ushort_as_half((unsigned short)(w & 0xFFFF)));
}
__device__ __forceinline__ float wd_h2f_hi(uint32_t w) {
  return __half2float(__ushort_as_half((unsigned short)(w >> 16)));
}
__device__ __forceinline__ uint32_t wd_sc2(uint32_t lo4, uint32_t hi4, int s) {
  const uint32_t w = s < 4 ? lo4 : hi4;
  const uint32_t k = s & 3;
  return hsub2_u32(prmt(w, 0x64646464u, 0x5040u | k | (k << 8)), 0x64006400u);
}
__device__ __forceinline__ float wd_sbyte(uint4 v, int k) {
  const uint32_t w = k < 4 ? v.x : k < 8 ? v.y : k < 12 ? v.z : v.w;
  return (float)(int8_t)((w >> (8 * (k & 3))) & 0xFF);
}

// This lane's view of the unit's prepared activations, per MMA group.
template <int NMG>
struct WdX {
  const uint8_t* f[NMG];   // fragments of 32-column group 0 (stride fs[mg])
  uint32_t fs[NMG];
  uint32_t xs[NMG];        // Q4_K sub-block sum word
  float inv[NMG];          // inverse activation scale of batch row 4 mg + (lane & 3)
};

// Two tiles (w[0], w[1]; w[1] may be absent) of one Q4_K unit: tg / tg8 +=
// rows g / g + 8, batch rows 4 mg + t.
template <int NMG, int T>
__device__ __forceinline__ void wd_q4k(const uint8_t* const (&w)[T], int nt, const WdX<NMG>& X, int lane,
                                       float (&tg)[T][NMG], float (&tg8)[T][NMG]) {
  const int g = lane >> 2, t = lane & 3;
  uint32_t scl0[T], sch0[T], scl1[T], sch1[T];
  float d0[T], d1[T];
  float C[T][NMG][4];
#pragma unroll
  for (int tt = 0; tt < T; tt++) {
#pragma unroll
    for (int mg = 0; mg < NMG; mg++)
#pragma unroll
      for (int i = 0; i < 4; i++) C[tt][mg][i] = 0.f;
    if (tt >= nt) continue;
    const uint4 h0 = *(const uint4*)(w[tt] + 16 * g), h1 = *(const uint4*)(w[tt] + 16 * (g + 8));
    scl0[tt] = h0.y & 0x3F3F3F3Fu;
    sch0[tt] = (h0.w & 0x0F0F0F0Fu) | ((h0.y >> 2) & 0x30303030u);
    scl1[tt] = h1.y & 0x3F3F3F3Fu;
    sch1[tt] = (h1.w & 0x0F0F0F0Fu) | ((h1.y >> 2) & 0x30303030u);
    const uint32_t mnl0 = h0.z & 0x3F3F3F3Fu, mnh0 = ((h0.w >> 4) & 0x0F0F0F0Fu) | ((h0.z >> 2) & 0x30303030u);
    const uint32_t mnl1 = h1.z & 0x3F3F3F3Fu, mnh1 = ((h1.w >> 4) & 0x0F0F0F0Fu) | ((h1.z >> 2) & 0x30303030u);
    d0[tt] = wd_h2f_lo(h0.x) * 16777216.f;
    d1[tt] = wd_h2f_lo(h1.x) * 1048576.f;
    const float dm0 = wd_h2f_hi(h0.x) * 32.f, dm1 = wd_h2f_hi(h1.x) * 32.f;
    // mins: A[row][k] = m_k(row) for k < 8, B[k][col] = X_k(col) 2^-5
    const uint32_t msel = (t & 1) ? 0x5342u : 0x5140u;
    const uint32_t am0 = hsub2_u32(prmt(t < 2 ? mnl0 : mnh0, 0x64646464u, msel), 0x64006400u);
    const uint32_t am1 = hsub2_u32(prmt(t < 2 ? mnl1 : mnh1, 0x64646464u, msel), 0x64006400u);
#pragma unroll
    for (int mg = 0; mg < NMG; mg++) {  // the mins' share goes into the sums straight away
      float Cm[4] = {0.f, 0.f, 0.f, 0.f};
      mma16816(Cm, am0, am1, 0u, 0u, X.xs[mg], 0u);
      tg[tt][mg] -= X.inv[mg] * (dm0 * (Cm[0] + Cm[1]));
      tg8[tt][mg] -= X.inv[mg] * (dm1 * (Cm[2] + Cm[3]));
    }
  }
#pragma unroll
  for (int c = 0; c < 4; c++) {
    uint4 q[T];
#pragma unroll
    for (int tt = 0; tt < T; tt++)
      q[tt] = tt < nt ? *(const uint4*)(w[tt] + 256 + c * 512 + lane * 16) : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int hs = 0; hs < 2; hs++) {
      uint4 xv[NMG];
#pragma unroll
      for (int mg = 0; mg < NMG; mg++) xv[mg] = *(const uint4*)(X.f[mg] + (2 * c + hs) * X.fs[mg]);
      const int s = 2 * c + hs;
#pragma unroll
      for (int tt = 0; tt < T; tt++) {
        if (tt >= nt) continue;
        const uint32_t sg = wd_sc2(scl0[tt], sch0[tt], s), sg8 = wd_sc2(scl1[tt], sch1[tt], s);
#pragma unroll
        for (int kk = 0; kk < 2; kk++) {
          const int i = 2 * hs + kk;
          const uint32_t wv = i == 0 ? q[tt].x : i == 1 ? q[tt].y : i == 2 ? q[tt].z : q[tt].w;
          const uint32_t w8 = wv >> 8;
          const uint32_t a0 = hmul2_u32(wv & 0x000F000Fu, sg);
          const uint32_t a1 = hmul2_u32(wv & 0x00F000F0u, sg8);
          const uint32_t a2 = hmul2_u32(w8 & 0x000F000Fu, sg);
          const uint32_t a3 = hmul2_u32(w8 & 0x00F000F0u, sg8);
#pragma unroll
          for (int mg = 0; mg < NMG; mg++)
            mma16816(C[tt][mg], a0, a1, a2, a3, kk ? xv[mg].z : xv[mg].x, kk ? xv[mg].w : xv[mg].y);
        }
      }
    }
  }
#pragma unroll
  for (int tt = 0; tt < T; tt++) {
    if (tt >= nt) continue;
#pragma unroll
    for (int mg = 0; mg < NMG; mg++) {
      tg[tt][mg] += X.inv[mg] * (d0[tt] * (C[tt][mg][0] + C[tt][mg][1]));
      tg8[tt][mg] += X.inv[mg] * (d1[tt] * (C[tt][mg][2] + C[tt][mg][3]));
    }
  }
}

// Two tiles of one Q6_K unit (the per-16-column int8 scales applied to each
// MMA's result).
template <int NMG, int T>
__device__ __forceinline__ void wd_q6k(const uint8_t* const (&w)[T], int nt, const WdX<NMG>& X, int lane,
                                       float (&tg)[T][NMG], float (&tg8)[T][NMG]) {
  const int g = lane >> 2;
  uint4 s0[T], s1[T];
  float acc[T][NMG], acc8[T][NMG];
#pragma unroll
  for (int tt = 0; tt < T; tt++) {
#pragma unroll
    for (int mg = 0; mg < NMG; mg++) acc[tt][mg] = acc8[tt][mg] = 0.f;
    s0[tt] = s1[tt] = make_uint4(0, 0, 0, 0);
    if (tt >= nt) continue;
    s0[tt] = *(const uint4*)(w[tt] + 3072 + 16 * g);
    s1[tt] = *(const uint4*)(w[tt] + 3072 + 16 * (g + 8));
  }
#pragma unroll
  for (int c = 0; c < 4; c++) {
    uint4 Lq[T];
    uint2 Hq[T];
#pragma unroll
    for (int tt = 0; tt < T; tt++) {
      Lq[tt] = make_uint4(0, 0, 0, 0);
      Hq[tt] = make_uint2(0, 0);
      if (tt >= nt) continue;
      Lq[tt] = *(const uint4*)(w[tt] + c * 768 + lane * 16);
      Hq[tt] = *(const uint2*)(w[tt] + c * 768 + 512 + lane * 8);
    }
#pragma unroll
    for (int hs = 0; hs < 2; hs++) {
      uint4 xv[NMG];
#pragma unroll
      for (int mg = 0; mg < NMG; mg++) xv[mg] = *(const uint4*)(X.f[mg] + (2 * c + hs) * X.fs[mg]);
#pragma unroll
      for (int tt = 0; tt < T; tt++) {
        if (tt >= nt) continue;
#pragma unroll
        for (int kk = 0; kk < 2; kk++) {
          const int i = 2 * hs + kk, kt = 4 * c + i;
          const uint32_t L = i == 0 ? Lq[tt].x : i == 1 ? Lq[tt].y : i == 2 ? Lq[tt].z : Lq[tt].w;
          const uint32_t Hw = (i < 2 ? Hq[tt].x : Hq[tt].y) >> (2 * (i & 1));
          const uint32_t L8 = L >> 8, H8 = Hw >> 8, Hs = Hw << 8;
          const uint32_t a0 =
              hsub2_u32(lop3_and_or(L, 0x000F000Fu, lop3_and_or(Hw, 0x00300030u, 0x64006400u)), 0x64206420u);
          const uint32_t a1 =
              hsub2_u32(lop3_and_or(L, 0x00F000F0u, lop3_and_or(Hw, 0x03000300u, 0x64006400u)), 0x66006600u);
          const uint32_t a2 =
              hsub2_u32(lop3_and_or(L8, 0x000F000Fu, lop3_and_or(H8, 0x00300030u, 0x64006400u)), 0x64206420u);
          const uint32_t a3 =
              hsub2_u32(lop3_and_or(L8, 0x00F000F0u, lop3_and_or(Hs, 0x03000300u, 0x64006400u)), 0x66006600u);
          const float f0 = wd_sbyte(s0[tt], kt), f1 = wd_sbyte(s1[tt], kt);
#pragma unroll
          for (int mg = 0; mg < NMG; mg++) {
            float Cc[4] = {0.f, 0.f, 0.f, 0.f};
            mma16816(Cc, a0, a1, a2, a3, kk ? xv[mg].z : xv[mg].x, kk ? xv[mg].w : xv[mg].y);
            acc[tt][mg] += f0 * (Cc[0] + Cc[1]);
            acc8[tt][mg] += f1 * (Cc[2] + Cc[3]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int tt = 0; tt < T; tt++) {
    if (tt >= nt) continue;
    const uint32_t dp = *(const uint32_t*)(w[tt] + 3328 + 4 * g);
    const float d0 = wd_h2f_lo(dp), d1 = wd_h2f_hi(dp) * 0.0625f;
#pragma unroll
    for (int mg = 0; mg < NMG; mg++) {
      tg[tt][mg] += X.inv[mg] * d0 * acc[tt][mg];
      tg8[tt][mg] += X.inv[mg] * d1 * acc8[tt][mg];
    }
  }
}

template <int NT>
__device__ __forceinline__ void bar_sync_compute() { asm volatile("bar.sync 1, %0;" ::"n"(NT) : "memory"); }
__device__ __forceinline__ int64_t wd_first(int64_t c, int64_t n, int G) { return c * n / G; }
__device__ __forceinline__ int wd_owner(int64_t x, int64_t n, int G) {
  int c = (int)((x * G) / n);
  while (c + 1 < G && wd_first(c + 1, n, G) <= x) c++;
  while (c > 0 && wd_first(c, n, G) > x) c--;
  return c;
}
// Device scratch: partial sums [grid][2][16 tiles][4 groups][2][32] of row
// blocks split between CTAs, per-block arrival counters (zero between
// launches), the error word and the tensor-parallel epilogue's peers.
struct WdScratch {
  float* split;
  int* count;
  int* err;
  TpArgs tp;
};
constexpr int WD_SLOT = WD_TILES * 4 * 2 * 32;  // floats per partial row block

template <int QT, int EPI, int NMG, int T>
__global__ void __launch_bounds__(32 * (1 + WD_TILES / T), 1)
    k_qmv_wide(const uint8_t* __restrict__ W, int nunit, int64_t rows, int tiles, const uint8_t* __restrict__ xprep,
               int B, float* __restrict__ y, WdScratch scr) {
  using S = WideSmem<QT>;
  constexpr int CW = WD_TILES / T;  // compute warps
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* const gb = smem_raw + (base - smem_u32(smem_raw));
  const uint32_t full = base + S::BAR, empty = full + 8 * S::NS;
  volatile int* const last_flag = (volatile int*)(gb + S::MISC);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nrb = (tiles + WD_TILES - 1) / WD_TILES;
  const int64_t n = (int64_t)nrb * nunit;
  const int G = gridDim.x, cta = blockIdx.x;
  const int64_t i0 = wd_first(cta, n, G), i1 = wd_first(cta + 1, n, G);
  const int cnt = (int)(i1 - i0);
  if (threadIdx.x == 0) {
    for (int s = 0; s < S::NS; s++) {
      mbar_init(full + 8 * s, 1);
      mbar_init(empty + 8 * s, CW);  // the compute warps
    }
    mbar_fence_init();
  }
  for (int i = threadIdx.x; i < 1024 / 16; i += blockDim.x) *(uint4*)(gb + S::ZERO + 16 * i) = make_uint4(0, 0, 0, 0);
  __syncthreads();
  pdl_launch();
  pdl_wait();

  if (warp == 0) {  // producer: lane 0 waits and arms the stage; lanes 0..15 copy one tile unit each,
                    // lanes 16.. one activation group each
    const int nmg = (B + 3) >> 2;
    bool ok = true;
    int k = 0;
    for (; k < cnt; k++) {
      const int s = k % S::NS;
      bool go = true;
      if (lane == 0) go = k < S::NS || mbar_wait_bounded(empty + 8 * s, (uint32_t)((k / S::NS - 1) & 1));
      if (!__shfl_sync(0xFFFFFFFFu, go, 0)) {
        ok = false;
        break;
      }
      const int64_t it = i0 + k, rb = it / nunit, u = it % nunit;
      const int ntile = min(WD_TILES, tiles - (int)rb * WD_TILES);
      const uint32_t st = base + s * S::SB;
      if (lane == 0) {
        uint32_t xbytes = 0;
        for (int mg = 0; mg < nmg; mg++) xbytes += xunit_bytes(8 * min(4, B - 4 * mg));
        mbar_arrive_expect_tx(full + 8 * s, ntile * S::TBB + xbytes);
      }
      __syncwarp();
      if (lane < ntile) {
        bulk_g2s(st + lane * S::TBB, W + ((rb * WD_TILES + lane) * (int64_t)nunit + u) * S::TBB, S::TBB, full + 8 * s);
      } else if (lane >= 16 && lane < 16 + nmg) {
        const int mg = lane - 16, LW = 8 * min(4, B - 4 * mg);
        bulk_g2s(st + S::XOFF + mg * WD_XG, xprep + xprep_off(mg, nunit, (int)u, LW), xunit_bytes(LW), full + 8 * s);
      }
    }
    if (!ok && lane == 0) {  // no copy may still be writing when the block moves on
      atomicOr(scr.err, SI_DEVERR_WAIT_TIMEOUT);
      for (int j = max(0, k - S::NS); j < k; j++)
        mbar_wait_bounded(full + 8 * (j % S::NS), (uint32_t)((j / S::NS) & 1));
    }
  } else {
    const int cw = warp - 1, g = lane >> 2, t = lane & 3;
    bool ok = true;
    float tg[T][NMG], tg8[T][NMG];
#pragma unroll
    for (int tt = 0; tt < T; tt++)
#pragma unroll
      for (int mg = 0; mg < NMG; mg++) tg[tt][mg] = tg8[tt][mg] = 0.f;
    int64_t cur = i0 / nunit;
    // Write (or hand over) the sums of row block rb; every compute warp takes
    // the same steps, whatever failed.
    auto flush = [&](int64_t rb) {
      float v[T][NMG], v8[T][NMG];
#pragma unroll
      for (int tt = 0; tt < T; tt++)
#pragma unroll
        for (int mg = 0; mg < NMG; mg++) {
          v[tt][mg] = tg[tt][mg];
          v8[tt][mg] = tg8[tt][mg];
        }
      bool write = rb * nunit >= i0 && (rb + 1) * nunit <= i1;
      if (!write) {
        const int which = rb == i0 / nunit ? 0 : 1;
        float* sp = scr.split + ((int64_t)cta * 2 + which) * WD_SLOT;
#pragma unroll
        for (int tt = 0; tt < 2; tt++)
#pragma unroll
          for (int mg = 0; mg < NMG; mg++) {
            sp[(((T * cw + tt) * 4 + mg) * 2 + 0) * 32 + lane] = v[tt][mg];
            sp[(((T * cw + tt) * 4 + mg) * 2 + 1) * 32 + lane] = v8[tt][mg];
          }
        __threadfence();
        bar_sync_compute<CW * 32>();
        if (threadIdx.x == 32) {  // the first compute thread
          const int c_lo = wd_owner(rb * nunit, n, G), c_hi = wd_owner((rb + 1) * nunit - 1, n, G);
          const int old = atomicAdd(scr.count + rb, 1);
          const bool last = old == c_hi - c_lo;
          if (last) scr.count[rb] = 0;  // zero again for the next launch
          *last_flag = last ? 1 : 0;
        }
        bar_sync_compute<CW * 32>();
        write = *last_flag != 0;
        if (write) {
          __threadfence();
          const int c_lo = wd_owner(rb * nunit, n, G), c_hi = wd_owner((rb + 1) * nunit - 1, n, G);
#pragma unroll
          for (int tt = 0; tt < T; tt++)
#pragma unroll
            for (int mg = 0; mg < NMG; mg++) v[tt][mg] = v8[tt][mg] = 0.f;
          for (int c = c_lo; c <= c_hi; c++) {
            const int wch = rb == wd_first(c, n, G) / nunit ? 0 : 1;
            const float* cp = scr.split + ((int64_t)c * 2 + wch) * WD_SLOT;
#pragma unroll
            for (int tt = 0; tt < T; tt++)
#pragma unroll
              for (int mg = 0; mg < NMG; mg++) {
                v[tt][mg] += __ldcg(cp + (((T * cw + tt) * 4 + mg) * 2 + 0) * 32 + lane);
                v8[tt][mg] += __ldcg(cp + (((T * cw + tt) * 4 + mg) * 2 + 1) * 32 + lane);
              }
          }
        }
        bar_sync_compute<CW * 32>();  // the flag is read before a later block sets it
      }
      if (!write || !ok) return;
#pragma unroll
      for (int tt = 0; tt < T; tt++)
#pragma unroll
        for (int mg = 0; mg < NMG; mg++) {
          const int b = 4 * mg + t;
          if (b >= B) continue;
          const int64_t r0 = rb * (16 * WD_TILES) + 16 * (T * cw + tt) + g, r1 = r0 + 8;
          if (EPI == SI_EPI_TP) {
            const unsigned tag = scr.tp.tag();
            for (int p = 0; p < scr.tp.tp; p++) {
              uint2* yb = (uint2*)(scr.tp.peers[p] + scr.tp.slot_off) + (int64_t)b * scr.tp.ld;
              if (r0 < rows) st_tagged(yb + r0, __float_as_uint(v[tt][mg]), tag);
              if (r1 < rows) st_tagged(yb + r1, __float_as_uint(v8[tt][mg]), tag);
            }
          } else {
            float* yb = y + (int64_t)b * rows;
            if (r0 < rows) {
              if (EPI == SI_EPI_ADD) yb[r0] += v[tt][mg];
              else yb[r0] = v[tt][mg];
            }
            if (r1 < rows) {
              if (EPI == SI_EPI_ADD) yb[r1] += v8[tt][mg];
              else yb[r1] = v8[tt][mg];
            }
          }
        }
    };
    for (int k = 0; k < cnt; k++) {
      const int s = k % S::NS;
      const int64_t it = i0 + k, rb = it / nunit;
      if (rb != cur) {
        flush(cur);
#pragma unroll
        for (int tt = 0; tt < T; tt++)
#pragma unroll
          for (int mg = 0; mg < NMG; mg++) tg[tt][mg] = tg8[tt][mg] = 0.f;
        cur = rb;
      }
      if (ok && !mbar_wait_bounded(full + 8 * s, (uint32_t)((k / S::NS) & 1))) {
        ok = false;
        if (lane == 0) atomicOr(scr.err, SI_DEVERR_WAIT_TIMEOUT);
      }
      if (!ok) continue;
      const int ntile = min(WD_TILES, tiles - (int)rb * WD_TILES);
      if (T * cw < ntile) {
        const uint8_t* st = gb + s * S::SB;
        WdX<NMG> X;
#pragma unroll
        for (int mg = 0; mg < NMG; mg++) {
          const int LW = 8 * min(4, B - 4 * mg);
          const uint8_t* xu = st + S::XOFF + mg * WD_XG;
          const bool on = lane < LW;
          X.f[mg] = on ? xu + lane * 16 : gb + S::ZERO;
          X.fs[mg] = on ? (uint32_t)(LW * 16) : 0u;
          X.xs[mg] = on ? *(const uint32_t*)(xu + 8 * LW * 16 + lane * 4) : 0u;
          X.inv[mg] = 8 * t < LW ? *(const float*)(xu + 132 * LW + 4 * t) : 0.f;
        }
        const uint8_t* w[T];
#pragma unroll
        for (int tt = 0; tt < T; tt++) w[tt] = st + (T * cw + tt) * S::TBB;
        const int nt = min(T, ntile - T * cw);
        if (QT == SI_Q4_K) wd_q4k<NMG, T>(w, nt, X, lane, tg, tg8);
        else wd_q6k<NMG, T>(w, nt, X, lane, tg, tg8);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty + 8 * s);
    }
    flush(cur);
  }
  __syncthreads();
}

template <int QT, int EPI, int NMG, int T>
int launch_wide_k(cudaStream_t s, const si_weight* w, const uint8_t* xprep, int B, float* y, const WdScratch& scr,
                  int sms, bool pdl) {
  using S = WideSmem<QT>;
  static DeviceOnce attr_set;
  int dev = 0;
  SI_CUDA(cudaGetDevice(&dev));
  if (!attr_set.done(dev)) {
    SI_CUDA(cudaFuncSetAttribute(k_qmv_wide<QT, EPI, NMG, T>, cudaFuncAttributeMaxDynamicSharedMemorySize, S::SMEM));
    attr_set.mark(dev);
  }
  const int64_t n = ((w->tiles + WD_TILES - 1) / WD_TILES) * w->nblk;
  const int G = (int)std::min<int64_t>(sms, n);
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(G);
  cfg.blockDim = dim3(32 * (1 + WD_TILES / T));
  cfg.dynamicSmemBytes = S::SMEM;
  cfg.stream = s;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  SI_CUDA(cudaLaunchKernelEx(&cfg, k_qmv_wide<QT, EPI, NMG, T>, (const uint8_t*)w->dev, (int)w->nblk, w->rows,
                             (int)w->tiles, xprep, B, y, scr));
  return SI_OK;
}

template <int QT, int EPI>
int launch_wide_q(cudaStream_t s, const si_weight* w, const uint8_t* xprep, int B, float* y, const WdScratch& scr,
                  int sms, bool pdl) {
  static const int tsel = [] {  // tiles per compute warp: SHARPINFER_B200_QMV_WIDE_T=2 selects two
    const char* e = getenv("SHARPINFER_B200_QMV_WIDE_T");
    return e ? atoi(e) : 0;
  }();
  const bool t2 = tsel == 2;  // one tile per warp measured faster at every batch
  if (B <= 8)
    return t2 ? launch_wide_k<QT, EPI, 2, 2>(s, w, xprep, B, y, scr, sms, pdl)
              : launch_wide_k<QT, EPI, 2, 1>(s, w, xprep, B, y, scr, sms, pdl);
  if (B <= 12)
    return t2 ? launch_wide_k<QT, EPI, 3, 2>(s, w, xprep, B, y, scr, sms, pdl)
              : launch_wide_k<QT, EPI, 3, 1>(s, w, xprep, B, y, scr, sms, pdl);
  return t2 ? launch_wide_k<QT, EPI, 4, 2>(s, w, xprep, B, y, scr, sms, pdl)
            : launch_wide_k<QT, EPI, 4, 1>(s, w, xprep, B, y, scr, sms, pdl);
}

template <int EPI>
int launch_wide_e(cudaStream_t s, const si_weight* w, const uint8_t* xprep, int B, float* y, const WdScratch& scr,
                  int sms, bool pdl) {
  if (w->qtype == SI_Q4_K) return launch_wide_q<SI_Q4_K, EPI>(s, w, xprep, B, y, scr, sms, pdl);
  return launch_wide_q<SI_Q6_K, EPI>(s, w, xprep, B, y, scr, sms, pdl);
}

}  // namespace

bool qmv_wide_enabled() {
  const char* e = getenv("SHARPINFER_B200_QMV_WIDE");
  return !(e && e[0] == '0');
}

size_t qmv_wide_split_bytes(int sms) { return (size_t)sms * 2 * WD_SLOT * sizeof(float); }

int launch_qmv_wide(cudaStream_t s, const si_weight* w, const uint8_t* xprep, int B, float* y, int epi,
                    const QmvBuffers& qb, bool pdl) {
  if ((w->qtype != SI_Q4_K && w->qtype != SI_Q6_K) || B < 5 || B > 16 || ((uintptr_t)xprep & 15)) return -1;
  // Below 448 row tiles (7168 rows) the one-tile-per-CTA kernel is faster on
  // B200: its 8-warp CTAs spread over every SM, where this kernel leaves most
  // CTAs with one or two row blocks.  SHARPINFER_B200_QMV_WIDE=2 forces this kernel.
  const char* e = getenv("SHARPINFER_B200_QMV_WIDE");
  if (w->tiles < 448 && !(e && e[0] == '2')) return -1;
  if (qmv_wide_split_bytes(qb.sms) > qb.split_bytes || (w->tiles + WD_TILES - 1) / WD_TILES > qb.count_n) return -1;
  const WdScratch scr{qb.split, qb.count, qb.err, qb.tp};
  if (epi == SI_EPI_ADD) return launch_wide_e<SI_EPI_ADD>(s, w, xprep, B, y, scr, qb.sms, pdl);
  if (epi == SI_EPI_TP) return launch_wide_e<SI_EPI_TP>(s, w, xprep, B, y, scr, qb.sms, pdl);
  return launch_wide_e<SI_EPI_STORE>(s, w, xprep, B, y, scr, qb.sms, pdl);
}

}  // namespace si
