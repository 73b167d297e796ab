// Q4_K matvec for batch 5..16 on the 5th-generation tensor cores.
//
// y[b][r] = sum_c W[r][c] x[b][c] with W in the repacked Q4_K layout (16-row
// tiles, 2304-byte units of 16 rows x 256 columns) and x in the prepared
// activation format (per 256-column unit and group of 4 batch rows: f16
// hi + lo fragments, Q4_K sub-block sums, inverse scales).
//
// Work item = 128 rows (8 tiles) x one 256-column unit.  The items, numbered
// row-block-major, are split into one contiguous range per persistent CTA.
// Per item:
//   - warp 0 bulk-copies the 8 weight units and the unit's prepared
//     activations into a 4-stage shared-memory ring;
//   - warps 2..9 (one 16-row tile each) turn the 4-bit quants into f16
//     sc * q (exact: the nibble masked in place is the subnormal q 2^-24,
//     times the 6-bit scale) and store them with tcgen05.st straight into a
//     tensor-memory A operand (128 lanes = rows, K along columns), plus the
//     6-bit mins; they also rearrange the activation fragments into the
//     shared-memory B operand (N = 2 x batch columns: hi and lo);
//   - warp 1 issues 16 tcgen05.mma (M 128, N 16/32, K 16; A from tensor
//     memory) for the scaled quants and one for the mins, into a
//     double-buffered accumulator;
//   - warps 10..13 read the accumulators (lane = row) and add
//     inv_b (d (hi + lo) - dmin (mins_hi + mins_lo)) into per-row sums.
// The tensor core reads only the small B tile from shared memory, so the
// shared-memory bandwidth goes to the ring and the rearrangement.
//
// The K order inside each MMA is permuted the same way on both operands:
// MMA position 4t + {0,1,2,3} holds original columns {2t, 2t+1, 2t+8, 2t+9}
// of the 16-column step, which is the order in which both the weight
// fragments and the activation fragments already sit in memory.
//
// A row block whose units lie in two or more CTAs' ranges is finished by the
// last of them to arrive (per-block counter), adding the others' partial sums
// in CTA order; the result does not depend on timing.
#include "common.cuh"
#include "prepfmt.cuh"
#include "tcgen05.cuh"

#include <cstdlib>
#include <algorithm>

namespace si {
namespace {

constexpr int TC_THREADS = 14 * 32;   // producer, MMA, 8 converters, 4 epilogue
constexpr int TC_NS = 4;              // weight/activation ring stages
constexpr int TC_UNIT = 2304;         // repacked Q4_K unit (16 rows x 256)
constexpr int TC_WB = 8 * TC_UNIT;    // weights of one item
constexpr int TC_XG = 132 * 32 + 16;  // prepared activations of one unit, one full group
constexpr int TC_XB = 4 * TC_XG;      // ... all four groups
constexpr int TC_SB = TC_WB + TC_XB;  // ring stage
constexpr int TC_BT = 32 * 32 * 16;   // B operand of one unit: 16 steps x (32 rows x 16 f16)
constexpr int TC_BM = 32 * 32;        // B operand of the mins: 32 rows x 16 f16
// TMEM columns: A buffers at 136 a (+128: mins), accumulators at 272 + 64 c (+32: mins)
constexpr uint32_t TC_TMEM_COLS = 512;

// Shared-memory map (offsets from a 1024-aligned base).
constexpr int OFF_RING = 0;
constexpr int OFF_BT = OFF_RING + TC_NS * TC_SB;      // [2] B tiles
constexpr int OFF_BM = OFF_BT + 2 * TC_BT;            // [2] B of the mins
constexpr int OFF_SC = OFF_BM + 2 * TC_BM;            // [2][128] float2 (d', dmin')
constexpr int OFF_INV = OFF_SC + 2 * 128 * 8;         // [2][16] float
constexpr int OFF_BAR = OFF_INV + 2 * 16 * 4;         // barriers
constexpr int OFF_MISC = OFF_BAR + 8 * (2 * TC_NS + 9);
constexpr int TC_SMEM = OFF_MISC + 16 + 1024;         // + alignment slack

__device__ __forceinline__ uint64_t sdesc_plain(uint32_t saddr) {
  // K-major, no swizzle: core matrices of 8 rows x 16 B; LBO 128 B (next 8
  // columns of K), SBO 256 B (next 8 rows), descriptor version 1.
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(256 >> 4) << 32) |
         ((uint64_t)1 << 46);
}

__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t b, uint32_t idesc,
                                            uint32_t acc) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p; }" ::"r"(
          tmem_d),
      "r"(tmem_a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// 16 lanes x 8 columns per repetition; thread (g, t): r0 lane g column 2t,
// r1 lane g column 2t + 1, r2 / r3 the same for lane g + 8.
__device__ __forceinline__ void tmem_st16x256_x4(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.16x256b.x4.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st16x256_x1(uint32_t taddr, uint32_t r0, uint32_t r1, uint32_t r2,
                                                 uint32_t r3) {
  asm volatile("tcgen05.st.sync.aligned.16x256b.x1.b32 [%0], {%1,%2,%3,%4};" ::"r"(taddr), "r"(r0), "r"(r1),
               "r"(r2), "r"(r3)
               : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_ld32x32_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void bar_sync_epi() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Item range of CTA c of G over n items.
__device__ __forceinline__ int64_t tc_first(int64_t c, int64_t n, int G) { return c * n / G; }

// Device scratch: partial sums [grid][2][16][128] of row blocks split
// between CTAs, per-block arrival counters (zero between launches), the
// error word and the tensor-parallel epilogue's peers.
struct TcScratch {
  float* split;
  int* count;
  int* err;
  TpArgs tp;
};

// CTA holding item x (the ranges are c n / G .. (c + 1) n / G, none empty).
__device__ __forceinline__ int tc_owner(int64_t x, int64_t n, int G) {
  int c = (int)((x * G) / n);
  while (c + 1 < G && tc_first(c + 1, n, G) <= x) c++;
  while (c > 0 && tc_first(c, n, G) > x) c--;
  return c;
}

__device__ __forceinline__ float h2f_lo(uint32_t w) {
  return __half2float(__ushort_as_half((unsigned short)(w & 0xFFFF)));
}
__device__ __forceinline__ float h2f_hi(uint32_t w) {
  return __half2float(__ushort_as_half((unsigned short)(w >> 16)));
}

// (sc_s, sc_s) as f16x2 for sub-block s of a row's decoded 6-bit scales.
__device__ __forceinline__ uint32_t tc_sc2(uint32_t lo4, uint32_t hi4, int s) {
  const uint32_t w = s < 4 ? lo4 : hi4;
  const uint32_t k = s & 3;
  return hsub2_u32(prmt(w, 0x64646464u, 0x5040u | k | (k << 8)), 0x64006400u);
}

// One 16-row Q4_K unit (raw, shared memory) into tensor memory: quants of
// step 4c + i at columns 32c + 8i of `ta` (lanes g, g + 8 of the tile), the
// mins at column 128.  Returns the rows' (d', dmin') for lanes g and g + 8.
__device__ __forceinline__ void tc_convert_unit(const uint8_t* wu, uint32_t ta, int lane, float2& s0, float2& s1) {
  const int g = lane >> 2, t = lane & 3;
  const uint4 h0 = *(const uint4*)(wu + 16 * g), h1 = *(const uint4*)(wu + 16 * (g + 8));
  const uint32_t scl0 = h0.y & 0x3F3F3F3Fu, mnl0 = h0.z & 0x3F3F3F3Fu;
  const uint32_t sch0 = (h0.w & 0x0F0F0F0Fu) | ((h0.y >> 2) & 0x30303030u);
  const uint32_t mnh0 = ((h0.w >> 4) & 0x0F0F0F0Fu) | ((h0.z >> 2) & 0x30303030u);
  const uint32_t scl1 = h1.y & 0x3F3F3F3Fu, mnl1 = h1.z & 0x3F3F3F3Fu;
  const uint32_t sch1 = (h1.w & 0x0F0F0F0Fu) | ((h1.y >> 2) & 0x30303030u);
  const uint32_t mnh1 = ((h1.w >> 4) & 0x0F0F0F0Fu) | ((h1.z >> 2) & 0x30303030u);
#pragma unroll
  for (int c = 0; c < 4; c++) {
    const uint4 q = *(const uint4*)(wu + 256 + c * 512 + lane * 16);
    uint32_t r[16];
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int s = 2 * c + (i >> 1);
      const uint32_t sg = tc_sc2(scl0, sch0, s), sg8 = tc_sc2(scl1, sch1, s);
      const uint32_t w = i == 0 ? q.x : i == 1 ? q.y : i == 2 ? q.z : q.w;
      const uint32_t w8 = w >> 8;
      // nibble masked in place = f16 subnormal q 2^-24 (16 q 2^-24 for row g + 8)
      r[4 * i + 0] = hmul2_u32(w & 0x000F000Fu, sg);     // row g,     k 2t, 2t+1
      r[4 * i + 1] = hmul2_u32(w8 & 0x000F000Fu, sg);    // row g,     k 2t+8, 2t+9
      r[4 * i + 2] = hmul2_u32(w & 0x00F000F0u, sg8);    // row g + 8, k 2t, 2t+1
      r[4 * i + 3] = hmul2_u32(w8 & 0x00F000F0u, sg8);   // row g + 8, k 2t+8, 2t+9
    }
    tmem_st16x256_x4(ta + 32 * c, r);
  }
  // mins: positions 4t, 4t+1 = m_2t, m_2t+1; positions 4t+2, 4t+3 = 0
  const uint32_t msel = (t & 1) ? 0x5342u : 0x5140u;
  const uint32_t am0 = hsub2_u32(prmt(t < 2 ? mnl0 : mnh0, 0x64646464u, msel), 0x64006400u);
  const uint32_t am1 = hsub2_u32(prmt(t < 2 ? mnl1 : mnh1, 0x64646464u, msel), 0x64006400u);
  tmem_st16x256_x1(ta + 128, am0, 0u, am1, 0u);
  s0 = make_float2(h2f_lo(h0.x) * 16777216.f, h2f_hi(h0.x) * 32.f);
  s1 = make_float2(h2f_lo(h1.x) * 1048576.f, h2f_hi(h1.x) * 32.f);
}

template <int EPI, int NB>
__global__ void __launch_bounds__(TC_THREADS, 1)
    k_qmv_tc(const uint8_t* __restrict__ W, int nunit, int64_t rows, int tiles, const uint8_t* __restrict__ xprep,
             int B, float* __restrict__ y, TcScratch scr) {
  constexpr uint32_t IDESC = (1u << 4) | ((uint32_t)(NB >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* const gb = smem_raw + (base - smem_u32(smem_raw));
  const uint32_t bar = base + OFF_BAR;
  // barriers: full[4] empty[4] abfull[2] abempty[2] accfull[2] accempty[2] done
  const uint32_t full = bar, empty = bar + 8 * TC_NS, abfull = bar + 16 * TC_NS, abempty = abfull + 16,
                 accfull = abempty + 16, accempty = accfull + 16, done = accempty + 16;
  volatile int* const abort_flag = (volatile int*)(gb + OFF_MISC);
  volatile int* const last_flag = (volatile int*)(gb + OFF_MISC + 4);
  const uint32_t tslot = base + OFF_MISC + 8;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nrb = (tiles + 7) / 8;
  const int64_t n = (int64_t)nrb * nunit;
  const int G = gridDim.x, cta = blockIdx.x;
  const int64_t i0 = tc_first(cta, n, G), i1 = tc_first(cta + 1, n, G);
  const int cnt = (int)(i1 - i0);
  const int nmg = (B + 3) >> 2;

  if (threadIdx.x == 0) {
    for (int s = 0; s < TC_NS; s++) {
      mbar_init(full + 8 * s, 1);
      mbar_init(empty + 8 * s, 8);
    }
    for (int a = 0; a < 2; a++) {
      mbar_init(abfull + 8 * a, 8);
      mbar_init(abempty + 8 * a, 1);
      mbar_init(accfull + 8 * a, 1);
      mbar_init(accempty + 8 * a, 4);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  // B operands start zeroed: columns past 2 B and positions 4t+2, 4t+3 of the
  // mins stay zero.
  for (int i = threadIdx.x; i < (2 * TC_BT + 2 * TC_BM) / 16; i += TC_THREADS)
    *(uint4*)(gb + OFF_BT + 16 * i) = make_uint4(0, 0, 0, 0);
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tslot),
                 "r"(TC_TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = lds_u32(tslot);
  pdl_launch();
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {  // producer
      bool ok = true;
      int k = 0;
      for (; k < cnt; k++) {
        const int s = k % TC_NS;
        if (*abort_flag) { ok = false; break; }
        if (k >= TC_NS && !mbar_wait_bounded(empty + 8 * s, (uint32_t)((k / TC_NS - 1) & 1))) { ok = false; break; }
        const int64_t it = i0 + k, rb = it / nunit, u = it % nunit;
        const int ntile = min(8, tiles - (int)rb * 8);
        uint32_t xbytes = 0;
        for (int mg = 0; mg < nmg; mg++) xbytes += xunit_bytes(8 * min(4, B - 4 * mg));
        const uint32_t st = base + OFF_RING + s * TC_SB;
        mbar_arrive_expect_tx(full + 8 * s, ntile * TC_UNIT + xbytes);
        for (int tt = 0; tt < ntile; tt++)
          bulk_g2s(st + tt * TC_UNIT, W + ((rb * 8 + tt) * (int64_t)nunit + u) * TC_UNIT, TC_UNIT, full + 8 * s);
        for (int mg = 0; mg < nmg; mg++) {
          const int LW = 8 * min(4, B - 4 * mg);
          bulk_g2s(st + TC_WB + mg * TC_XG, xprep + xprep_off(mg, nunit, (int)u, LW), xunit_bytes(LW), full + 8 * s);
        }
      }
      if (!ok) {  // no bulk copy may still be writing when the block moves on
        *abort_flag = 1;
        atomicOr(scr.err, SI_DEVERR_WAIT_TIMEOUT);
        for (int j = max(0, k - TC_NS); j < k; j++) mbar_wait_bounded(full + 8 * (j % TC_NS), (uint32_t)((j / TC_NS) & 1));
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      bool ok = true;
      for (int k = 0; k < cnt && ok; k++) {
        const int a = k & 1;
        if (*abort_flag || !mbar_wait_bounded(abfull + 8 * a, (uint32_t)((k >> 1) & 1)) ||
            (k >= 2 && !mbar_wait_bounded(accempty + 8 * a, (uint32_t)(((k >> 1) - 1) & 1)))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t ta = tmem + 136u * a, td = tmem + 272u + 64u * a;
        const uint32_t sb = base + OFF_BT + a * TC_BT;
#pragma unroll
        for (int st = 0; st < 16; st++) umma_f16_ts(td, ta + 8 * st, sdesc_plain(sb + st * 1024), IDESC, st > 0);
        umma_f16_ts(td + 32, ta + 128, sdesc_plain(base + OFF_BM + a * TC_BM), IDESC, 0);
        umma_commit(abempty + 8 * a);
        umma_commit(accfull + 8 * a);
      }
      umma_commit(done);
      if (!ok) {
        *abort_flag = 1;
        atomicOr(scr.err, SI_DEVERR_WAIT_TIMEOUT);
      }
      mbar_wait_bounded(done, 0);  // every MMA finished before the columns are freed
    }
  } else if (warp < 10) {  // converters: warp w owns tile 2 (w % 4) + (w - 2) / 4 of the block
    const int cw = warp - 2, q = warp & 3, tb = 2 * q + (cw >> 2);
    const int g = lane >> 2, t = lane & 3;
    float2* const scv = (float2*)(gb + OFF_SC);
    float* const invv = (float*)(gb + OFF_INV);
    bool ok = true;
    for (int k = 0; k < cnt; k++) {
      const int s = k % TC_NS, a = k & 1;
      if (*abort_flag || !mbar_wait_bounded(full + 8 * s, (uint32_t)((k / TC_NS) & 1)) ||
          (k >= 2 && (!mbar_wait_bounded(abempty + 8 * a, (uint32_t)(((k >> 1) - 1) & 1)) ||
                      !mbar_wait_bounded(accempty + 8 * a, (uint32_t)(((k >> 1) - 1) & 1))))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int64_t it = i0 + k, rb = it / nunit;
      const int ntile = min(8, tiles - (int)rb * 8);
      const uint8_t* st = gb + OFF_RING + s * TC_SB;
      if (tb < ntile) {
        float2 s0, s1;
        const uint32_t ta = tmem + ((uint32_t)(32 * q + 16 * (cw >> 2)) << 16) + 136u * a;
        tc_convert_unit(st + tb * TC_UNIT, ta, lane, s0, s1);
        if (t == 0) {
          scv[a * 128 + 16 * tb + g] = s0;
          scv[a * 128 + 16 * tb + g + 8] = s1;
        }
      }
      // activation fragments of 32-column group jj = cw -> steps 2 jj, 2 jj + 1
      uint8_t* const bt = gb + OFF_BT + a * TC_BT;
      for (int mg = 0; mg < nmg; mg++) {
        const int LW = 8 * min(4, B - 4 * mg);
        const uint8_t* xu = st + TC_WB + mg * TC_XG;
        if (lane < LW) {
          const uint4 f = *(const uint4*)(xu + (cw * LW + lane) * 16);
          const int nn = 8 * mg + (lane >> 2);
          const int off = ((t >> 1) * 128) + (nn >> 3) * 256 + (nn & 7) * 16 + (t & 1) * 8;
          *(uint2*)(bt + (2 * cw) * 1024 + off) = make_uint2(f.x, f.y);
          *(uint2*)(bt + (2 * cw + 1) * 1024 + off) = make_uint2(f.z, f.w);
          if (cw == mg) {  // the group's sub-block sums -> B of the mins
            const uint32_t sw = *(const uint32_t*)(xu + 8 * LW * 16 + lane * 4);
            *(uint2*)(gb + OFF_BM + a * TC_BM + off) = make_uint2(sw, 0u);
          }
          if (cw == 4 + mg && lane < LW / 8)  // inverse scales of the group's batch rows
            invv[a * 16 + 4 * mg + lane] = *(const float*)(xu + 132 * LW + 4 * lane);
        }
      }
      tmem_wait_st();
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(abfull + 8 * a);
        mbar_arrive(empty + 8 * s);
      }
    }
    if (!ok && lane == 0) {
      *abort_flag = 1;
      atomicOr(scr.err, SI_DEVERR_WAIT_TIMEOUT);
    }
  } else {  // epilogue: TMEM lanes 32 (warp % 4) .. + 31 = rows of the block
    const int q = warp & 3, r = 32 * q + lane;
    const float2* const scv = (const float2*)(gb + OFF_SC);
    const float* const invv = (const float*)(gb + OFF_INV);
    bool ok = true;
    float acc[16];
#pragma unroll
    for (int b = 0; b < 16; b++) acc[b] = 0.f;
    int64_t cur = i0 / nunit;
    // Write (or hand over) the sums of row block rb; every epilogue warp
    // takes the same steps, whatever failed.
    auto flush = [&](int64_t rb) {
      const int64_t row = rb * 128 + r;
      const bool whole = rb * nunit >= i0 && (rb + 1) * nunit <= i1;
      float v[16];
#pragma unroll
      for (int b = 0; b < 16; b++) v[b] = acc[b];
      bool write = whole;
      if (!whole) {
        const int which = rb == i0 / nunit ? 0 : 1;
        float* sp = scr.split + ((int64_t)cta * 2 + which) * 2048;
#pragma unroll
        for (int b = 0; b < 16; b++)
          if (b < B) sp[b * 128 + r] = v[b];
        __threadfence();
        bar_sync_epi();
        if (threadIdx.x == 10 * 32) {
          const int c_lo = tc_owner(rb * nunit, n, G), c_hi = tc_owner((rb + 1) * nunit - 1, n, G);
          const int old = atomicAdd(scr.count + rb, 1);
          const bool last = old == c_hi - c_lo;
          if (last) scr.count[rb] = 0;  // zero again for the next launch
          *last_flag = last ? 1 : 0;
        }
        bar_sync_epi();
        write = *last_flag != 0;
        if (write) {
          __threadfence();
          const int c_lo = tc_owner(rb * nunit, n, G), c_hi = tc_owner((rb + 1) * nunit - 1, n, G);
#pragma unroll
          for (int b = 0; b < 16; b++) v[b] = 0.f;
          for (int c = c_lo; c <= c_hi; c++) {
            const int w = rb == tc_first(c, n, G) / nunit ? 0 : 1;
            const float* cp = scr.split + ((int64_t)c * 2 + w) * 2048;
#pragma unroll
            for (int b = 0; b < 16; b++)
              if (b < B) v[b] += __ldcg(cp + b * 128 + r);
          }
        }
        bar_sync_epi();  // the flag is read before a later block sets it
      }
      if (write && ok && row < rows) {
        if (EPI == SI_EPI_TP) {
          const unsigned tag = scr.tp.tag();
          for (int p = 0; p < scr.tp.tp; p++) {
            uint2* yb = (uint2*)(scr.tp.peers[p] + scr.tp.slot_off);
#pragma unroll
            for (int b = 0; b < 16; b++)
              if (b < B) st_tagged(yb + (int64_t)b * scr.tp.ld + row, __float_as_uint(v[b]), tag);
          }
        } else {
#pragma unroll
          for (int b = 0; b < 16; b++)
            if (b < B) {
              float* dst = y + (int64_t)b * rows + row;
              if (EPI == SI_EPI_ADD) *dst += v[b];
              else *dst = v[b];
            }
        }
      }
    };
    for (int k = 0; k < cnt; k++) {
      const int a = k & 1;
      const int64_t rb = (i0 + k) / nunit;
      if (rb != cur) {
        flush(cur);
#pragma unroll
        for (int b = 0; b < 16; b++) acc[b] = 0.f;
        cur = rb;
      }
      if (ok && (*abort_flag || !mbar_wait_bounded(accfull + 8 * a, (uint32_t)((k >> 1) & 1)) ||
                 !mbar_wait_bounded(abfull + 8 * a, (uint32_t)((k >> 1) & 1)))) {
        ok = false;
        if (lane == 0) {
          *abort_flag = 1;
          atomicOr(scr.err, SI_DEVERR_WAIT_TIMEOUT);
        }
      }
      if (!ok) continue;
      tc_fence_after();
      uint32_t m[NB], mn[NB];
      const uint32_t td = tmem + ((uint32_t)(32 * q) << 16) + 272u + 64u * a;
      {
        uint32_t t16[16];
        tmem_ld32x32_x16(td, t16);
#pragma unroll
        for (int j = 0; j < 16; j++) m[j] = t16[j];
        tmem_ld32x32_x16(td + 32, t16);
#pragma unroll
        for (int j = 0; j < 16; j++) mn[j] = t16[j];
        if constexpr (NB == 32) {
          tmem_ld32x32_x16(td + 16, t16);
#pragma unroll
          for (int j = 0; j < 16; j++) m[16 + j] = t16[j];
          tmem_ld32x32_x16(td + 48, t16);
#pragma unroll
          for (int j = 0; j < 16; j++) mn[16 + j] = t16[j];
        }
      }
      const float2 sc = scv[a * 128 + r];
      float inv[NB / 2];
#pragma unroll
      for (int b = 0; b < NB / 2; b++) inv[b] = invv[a * 16 + b];
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(accempty + 8 * a);
#pragma unroll
      for (int b = 0; b < NB / 2; b++) {
        const float mm = __uint_as_float(m[2 * b]) + __uint_as_float(m[2 * b + 1]);
        const float mi = __uint_as_float(mn[2 * b]) + __uint_as_float(mn[2 * b + 1]);
        acc[b] += inv[b] * (sc.x * mm - sc.y * mi);
      }
    }
    flush(cur);
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TC_TMEM_COLS) : "memory");
  }
}

template <int EPI, int NB>
int launch_tc(cudaStream_t s, const si_weight* w, const uint8_t* xprep, int B, float* y, const TcScratch& scr,
              int sms, bool pdl) {
  static DeviceOnce attr_set;
  int dev = 0;
  SI_CUDA(cudaGetDevice(&dev));
  if (!attr_set.done(dev)) {
    SI_CUDA(cudaFuncSetAttribute(k_qmv_tc<EPI, NB>, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM));
    attr_set.mark(dev);
  }
  const int64_t n = ((w->tiles + 7) / 8) * w->nblk;
  const int G = (int)std::min<int64_t>(sms, n);
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(G);
  cfg.blockDim = dim3(TC_THREADS);
  cfg.dynamicSmemBytes = TC_SMEM;
  cfg.stream = s;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  SI_CUDA(cudaLaunchKernelEx(&cfg, k_qmv_tc<EPI, NB>, (const uint8_t*)w->dev, (int)w->nblk, w->rows, (int)w->tiles,
                             xprep, B, y, scr));
  return SI_OK;
}

}  // namespace

bool qmv_tc_enabled() {
  static const bool on = [] {
    const char* e = getenv("SHARPINFER_B200_QMV_TC");
    return !(e && e[0] == '0');
  }();
  return on;
}

size_t qmv_tc_split_bytes(int sms) { return (size_t)sms * 2 * 2048 * sizeof(float); }

int launch_qmv_tc(cudaStream_t s, const si_weight* w, const uint8_t* xprep, int B, float* y, int epi,
                  const QmvBuffers& qb, bool pdl) {
  if (w->qtype != SI_Q4_K || B < 5 || B > 16 || ((uintptr_t)xprep & 15)) return -1;
  if (qmv_tc_split_bytes(qb.sms) > qb.split_bytes || (w->tiles + 7) / 8 > qb.count_n) return -1;
  const TcScratch scr{qb.split, qb.count, qb.err, qb.tp};
  const bool n32 = B > 8;
  switch (epi) {
    case SI_EPI_ADD:
      return n32 ? launch_tc<SI_EPI_ADD, 32>(s, w, xprep, B, y, scr, qb.sms, pdl)
                 : launch_tc<SI_EPI_ADD, 16>(s, w, xprep, B, y, scr, qb.sms, pdl);
    case SI_EPI_TP:
      return n32 ? launch_tc<SI_EPI_TP, 32>(s, w, xprep, B, y, scr, qb.sms, pdl)
                 : launch_tc<SI_EPI_TP, 16>(s, w, xprep, B, y, scr, qb.sms, pdl);
    default:
      return n32 ? launch_tc<SI_EPI_STORE, 32>(s, w, xprep, B, y, scr, qb.sms, pdl)
                 : launch_tc<SI_EPI_STORE, 16>(s, w, xprep, B, y, scr, qb.sms, pdl);
  }
}

}  // namespace si
