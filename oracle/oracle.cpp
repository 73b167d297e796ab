// CPU ORACLE -- TEST INFRASTRUCTURE ONLY.
//
// A C++ restatement of SharpInfer's managed CPU path for the K-quant hot
// path.  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg
// load this library, and only as the checker (or the timed CPU baseline);
// nothing in the sharpinfer_b200 package links or calls it.
//
// Every function cites the reference file:line it follows (paths relative to
// the SharpInfer project root).  The reference is C# (.NET 8): RyuJIT does not
// contract a*b+c into FMA, and MathF.Exp/Pow/Sin/Cos/Sqrt map to the C
// runtime, so this file is compiled with -ffp-contract=off and uses glibc's
// expf/powf/sinf/cosf/sqrtf.
//
// Pinning: the dequantisers are checked bit for bit against gguf-py (the
// GGML reference Python implementation of the same block formats) and
// against known-answer blocks derived by hand from Quantization.cs.  The
// reference itself cannot be run here (C#, no .NET runtime, and its Models/
// directory is missing), so the f32 arithmetic below (dot-product lane order,
// norms, attention, decode step) is pinned only by this restatement.
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

#define OR_API extern "C" __attribute__((visibility("default")))

// QuantType values (Quantization.cs:6-22).
enum {
  QT_F32 = 0, QT_F16 = 1, QT_Q4_0 = 2, QT_Q8_0 = 8, QT_Q2_K = 10, QT_Q3_K = 11, QT_Q4_K = 12, QT_Q5_K = 13,
  QT_Q6_K = 14, QT_BF16 = 30
};

// ---------------------------------------------------------------------------
// Quantization.cs
// ---------------------------------------------------------------------------

// HalfToFloat (Quantization.cs:394-398): exact IEEE binary16 -> binary32.
OR_API float or_half_to_float(uint16_t h) {
  uint32_t sign = (uint32_t)(h >> 15) << 31;
  int exp = (h >> 10) & 0x1F;
  uint32_t man = h & 0x3FF;
  uint32_t bits;
  if (exp == 0x1F) {
    bits = sign | 0x7F800000u | (man << 13);
  } else if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {
      // subnormal: value = man * 2^-24, exact in binary32
      float v = (float)man * (1.0f / 16777216.0f);
      memcpy(&bits, &v, 4);
      bits |= sign;
    }
  } else {
    bits = sign | ((uint32_t)(exp - 15 + 127) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

static inline float half_at(const uint8_t* p) {
  return or_half_to_float((uint16_t)(p[0] | (p[1] << 8)));
}

// BlockSize / BlockBytes (Quantization.cs:31-65), the formats on this path.
OR_API int or_block_size(int qt) {
  switch (qt) {
    case QT_Q4_0: case QT_Q8_0: return 32;
    case QT_Q2_K: case QT_Q3_K: case QT_Q4_K: case QT_Q5_K: case QT_Q6_K: return 256;
    default: return 1;
  }
}
OR_API int or_block_bytes(int qt) {
  switch (qt) {
    case QT_Q4_0: return 18;
    case QT_Q8_0: return 34;
    case QT_Q2_K: return 84;
    case QT_Q3_K: return 110;
    case QT_Q4_K: return 144;
    case QT_Q5_K: return 176;
    case QT_Q6_K: return 210;
    case QT_F16: case QT_BF16: return 2;
    case QT_F32: return 4;
    default: return -1;
  }
}

// DequantQ8_0 (Quantization.cs:106-114): out[j] = (sbyte)q[j] * d.
static void dequant_q8_0_block(const uint8_t* b, float* out) {
  float scale = half_at(b);
  for (int j = 0; j < 32; j++) out[j] = (float)(int8_t)b[2 + j] * scale;
}

// GetScaleMinK4 (Quantization.cs:302-314).
static inline void get_scale_min_k4(int j, const uint8_t* q, uint8_t* sc, uint8_t* mn) {
  if (j < 4) {
    *sc = (uint8_t)(q[j] & 63);
    *mn = (uint8_t)(q[j + 4] & 63);
  } else {
    *sc = (uint8_t)((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4));
    *mn = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
  }
}

// DequantQ4_K (Quantization.cs:273-300).
static void dequant_q4_k_block(const uint8_t* b, float* out) {
  float d = half_at(b);
  float dmin = half_at(b + 2);
  const uint8_t* scales = b + 4;
  const uint8_t* qs = b + 16;
  int outIdx = 0, qIdx = 0;
  for (int j = 0; j < 8; j += 2) {
    uint8_t sc1, m1, sc2, m2;
    get_scale_min_k4(j, scales, &sc1, &m1);
    get_scale_min_k4(j + 1, scales, &sc2, &m2);
    float d1 = d * (float)sc1;
    float m1f = dmin * (float)m1;
    float d2 = d * (float)sc2;
    float m2f = dmin * (float)m2;
    for (int l = 0; l < 32; l++) {
      out[outIdx + l] = d1 * (float)(qs[qIdx + l] & 0xF) - m1f;
      out[outIdx + l + 32] = d2 * (float)(qs[qIdx + l] >> 4) - m2f;
    }
    outIdx += 64;
    qIdx += 32;
  }
}

// DequantQ6_K (Quantization.cs:362-391); the product is (d * sc) * (q - 32).
static void dequant_q6_k_block(const uint8_t* b, float* out) {
  const uint8_t* ql = b;
  const uint8_t* qh = b + 128;
  const int8_t* scales = (const int8_t*)(b + 192);
  float d = half_at(b + 208);
  int outIdx = 0;
  for (int n = 0; n < 2; n++) {
    int qlOff = n * 64, qhOff = n * 32, scOff = n * 8;
    for (int l = 0; l < 32; l++) {
      int scIdx = scOff + l / 16;
      int q1 = (ql[qlOff + l] & 0xF) | (((qh[qhOff + l] >> 0) & 3) << 4);
      int q2 = (ql[qlOff + l + 32] & 0xF) | (((qh[qhOff + l] >> 2) & 3) << 4);
      int q3 = (ql[qlOff + l] >> 4) | (((qh[qhOff + l] >> 4) & 3) << 4);
      int q4 = (ql[qlOff + l + 32] >> 4) | (((qh[qhOff + l] >> 6) & 3) << 4);
      out[outIdx + l] = d * (float)scales[scIdx] * (float)(q1 - 32);
      out[outIdx + l + 32] = d * (float)scales[scIdx + 2] * (float)(q2 - 32);
      out[outIdx + l + 64] = d * (float)scales[scIdx + 4] * (float)(q3 - 32);
      out[outIdx + l + 96] = d * (float)scales[scIdx + 6] * (float)(q4 - 32);
    }
    outIdx += 128;
  }
}

// DequantQ4_0 (Quantization.cs:71-83): out[j] = ((q & 0xF) - 8) * d,
// out[j + 16] = ((q >> 4) - 8) * d.
static void dequant_q4_0_block(const uint8_t* b, float* out) {
  float scale = half_at(b);
  for (int j = 0; j < 16; j++) {
    out[j] = (float)((b[2 + j] & 0x0F) - 8) * scale;
    out[j + 16] = (float)((b[2 + j] >> 4) - 8) * scale;
  }
}

// Q2_K, Q3_K and Q5_K in the GGML block layouts a GGUF file holds.  The
// reference's decoders (Quantization.cs:176-197, :205-267, :322-356) read
// these fields at other offsets -- restated as written further below -- so
// these follow the GGML layout, with the reference's arithmetic:
//   Q2_K [scales 16][qs 64][f16 d][f16 dmin]: element 128n + 32s + 16h + l =
//        (d * (sc & 15)) * ((qs[32n + 16h + l] >> 2s) & 3) - dmin * (sc >> 4),
//        sc = scales[8n + 2s + h]
//   Q3_K [hmask 32][qs 64][scales 12][f16 d]: the reference's scale unpacking
//        and loop (Quantization.cs:205-267) with d read from byte 108
//   Q5_K [f16 d][f16 dmin][scales 12][qh 32][qs 128]: the reference's loop
//        (Quantization.cs:322-356) with qh at byte 16 and qs at byte 48
static void dequant_q2_k_ggml(const uint8_t* b, float* out) {
  const uint8_t* scales = b;
  const uint8_t* qs = b + 16;
  float d = half_at(b + 80), dmin = half_at(b + 82);
  int outIdx = 0;
  for (int n = 0; n < 2; n++)
    for (int s = 0; s < 4; s++)
      for (int h = 0; h < 2; h++) {
        const uint8_t sc = scales[8 * n + 2 * s + h];
        float dl = d * (float)(sc & 0xF);
        float ml = dmin * (float)(sc >> 4);
        for (int l = 0; l < 16; l++) out[outIdx++] = dl * (float)((qs[32 * n + 16 * h + l] >> (2 * s)) & 3) - ml;
      }
}

static void q3_k_scales(const uint8_t* raw, int* scales) {
  for (int i = 0; i < 4; i++) {
    scales[i] = raw[i] & 0xF;
    scales[i + 4] = raw[i + 4] & 0xF;
    scales[i + 8] = raw[i] >> 4;
    scales[i + 12] = raw[i + 4] >> 4;
  }
  for (int i = 0; i < 4; i++) {
    uint8_t hi = raw[8 + i];
    scales[i] |= ((hi >> 0) & 3) << 4;
    scales[i + 4] |= ((hi >> 2) & 3) << 4;
    scales[i + 8] |= ((hi >> 4) & 3) << 4;
    scales[i + 12] |= ((hi >> 6) & 3) << 4;
  }
  for (int i = 0; i < 16; i++) scales[i] -= 32;
}

static void q3_k_body(float dAll, const uint8_t* hmask, const uint8_t* qs, const int* scales, float* out) {
  int outIdx = 0, qOff = 0, scIdx = 0;
  uint8_t m = 1;
  for (int n = 0; n < 2; n++) {
    int shift = 0;
    for (int j = 0; j < 4; j++) {
      float dl = dAll * (float)scales[scIdx];
      for (int l = 0; l < 16; l++) {
        int lo2 = (qs[qOff + l] >> shift) & 3, hb = (hmask[l] & m) ? 0 : -4;
        out[outIdx++] = dl * (float)(lo2 + hb);
      }
      float dl2 = dAll * (float)scales[scIdx + 1];
      for (int l = 16; l < 32; l++) {
        int lo2 = (qs[qOff + l] >> shift) & 3, hb = (hmask[l] & m) ? 0 : -4;
        out[outIdx++] = dl2 * (float)(lo2 + hb);
      }
      shift += 2;
      m = (uint8_t)(m << 1);
      scIdx += 2;
    }
    qOff += 32;
  }
}

static void dequant_q3_k_ggml(const uint8_t* b, float* out) {
  int scales[16];
  q3_k_scales(b + 96, scales);
  q3_k_body(half_at(b + 108), b, b + 32, scales, out);
}

static void q5_k_body(float d, float dmin, const uint8_t* scales, const uint8_t* qs, const uint8_t* qh, float* out) {
  int outIdx = 0, qIdx = 0, scIdx = 0;
  uint8_t u1 = 1, u2 = 2;
  for (int j = 0; j < 4; j++) {
    uint8_t sc1, m1, sc2, m2;
    get_scale_min_k4(scIdx, scales, &sc1, &m1);
    get_scale_min_k4(scIdx + 1, scales, &sc2, &m2);
    float d1 = d * (float)sc1, m1f = dmin * (float)m1, d2 = d * (float)sc2, m2f = dmin * (float)m2;
    for (int l = 0; l < 32; l++) {
      int hi1 = (qh[l] & u1) ? 16 : 0, hi2 = (qh[l] & u2) ? 16 : 0;
      out[outIdx + l] = d1 * (float)((qs[qIdx + l] & 0xF) + hi1) - m1f;
      out[outIdx + l + 32] = d2 * (float)((qs[qIdx + l] >> 4) + hi2) - m2f;
    }
    outIdx += 64;
    qIdx += 32;
    scIdx += 2;
    u1 = (uint8_t)(u1 << 2);
    u2 = (uint8_t)(u2 << 2);
  }
}

static void dequant_q5_k_ggml(const uint8_t* b, float* out) {
  q5_k_body(half_at(b), half_at(b + 2), b + 4, b + 48, b + 16, out);
}

// The reference's DequantQ2_K / DequantQ3_K / DequantQ5_K exactly as written
// (Quantization.cs:176-197, :205-267, :322-356): Q2_K reads [d][dmin][16
// scales][64 qs] and emits, for each scale j, the four 2-bit fields of
// qs[4j .. 4j + 3] in turn; Q3_K reads d from byte 0, hmask from 2, qs from
// 34 and the scales from 98; Q5_K reads qs from byte 16 and qh from 144.
// Kept to show where they part from the GGML layout above.
OR_API int or_dequant_reference_as_written(int qt, const uint8_t* data, int64_t nblocks, float* out) {
  for (int64_t i = 0; i < nblocks; i++) {
    float* o = out + i * 256;
    if (qt == QT_Q2_K) {
      const uint8_t* b = data + i * 84;
      float d = half_at(b), dmin = half_at(b + 2);
      const uint8_t* scales = b + 4;
      const uint8_t* qs = b + 20;
      int outIdx = 0;
      for (int j = 0; j < 16; j++) {
        float sc = d * (float)(scales[j] & 0xF), m = dmin * (float)(scales[j] >> 4);
        for (int l = 0; l < 4; l++) {
          uint8_t q = qs[j * 4 + l];
          o[outIdx++] = sc * (float)(q & 3) - m;
          o[outIdx++] = sc * (float)((q >> 2) & 3) - m;
          o[outIdx++] = sc * (float)((q >> 4) & 3) - m;
          o[outIdx++] = sc * (float)((q >> 6) & 3) - m;
        }
      }
    } else if (qt == QT_Q3_K) {
      const uint8_t* b = data + i * 110;
      int scales[16];
      q3_k_scales(b + 98, scales);
      q3_k_body(half_at(b), b + 2, b + 34, scales, o);
    } else if (qt == QT_Q5_K) {
      const uint8_t* b = data + i * 176;
      q5_k_body(half_at(b), half_at(b + 2), b + 4, b + 16, b + 144, o);
    } else {
      return -1;
    }
  }
  return 0;
}

// DequantizeTensor (Quantization.cs:415-469), restricted to the formats of
// this path.  Returns 0 on success, -1 for an unsupported type.
OR_API int or_dequant_tensor(int qt, const uint8_t* data, int64_t n, float* out) {
  if (qt == QT_F32) {
    memcpy(out, data, (size_t)n * 4);
    return 0;
  }
  if (qt == QT_F16) {
    for (int64_t i = 0; i < n; i++) out[i] = half_at(data + 2 * i);
    return 0;
  }
  if (qt == QT_BF16) {  // BFloat16ToFloat (Quantization.cs:404-409)
    for (int64_t i = 0; i < n; i++) {
      uint32_t bits = (uint32_t)(data[2 * i] | (data[2 * i + 1] << 8)) << 16;
      memcpy(&out[i], &bits, 4);
    }
    return 0;
  }
  int bs = or_block_size(qt), bb = or_block_bytes(qt);
  if (bs <= 1 || bb <= 0) return -1;
  int64_t nb = n / bs;
  for (int64_t b = 0; b < nb; b++) {
    const uint8_t* blk = data + b * bb;
    float* dst = out + b * bs;
    switch (qt) {
      case QT_Q8_0: dequant_q8_0_block(blk, dst); break;
      case QT_Q4_K: dequant_q4_k_block(blk, dst); break;
      case QT_Q6_K: dequant_q6_k_block(blk, dst); break;
      case QT_Q4_0: dequant_q4_0_block(blk, dst); break;
      case QT_Q2_K: dequant_q2_k_ggml(blk, dst); break;
      case QT_Q3_K: dequant_q3_k_ggml(blk, dst); break;
      case QT_Q5_K: dequant_q5_k_ggml(blk, dst); break;
      default: return -1;
    }
  }
  return 0;
}

// ---------------------------------------------------------------------------
// TensorOps.cs
// ---------------------------------------------------------------------------

// Dot (TensorOps.cs:20-57).  AVX path for n >= 8: eight lane accumulators,
// v[j] = v[j] + (a*b) with the product rounded first; then
// (hi + lo) -> s[0..3]; hadd -> (s0+s1), (s2+s3); result (s0+s1) + (s2+s3);
// then the scalar tail sum += a[i]*b[i].
OR_API float or_dot(const float* a, const float* b, int n) {
  float sum = 0.0f;
  int i = 0;
  if (n >= 8) {
    float v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (; i + 8 <= n; i += 8) {
      for (int j = 0; j < 8; j++) {
        float p = a[i + j] * b[i + j];
        v[j] = v[j] + p;
      }
    }
    float s0 = v[4] + v[0], s1 = v[5] + v[1], s2 = v[6] + v[2], s3 = v[7] + v[3];
    float h01 = s0 + s1, h23 = s2 + s3;
    sum = h01 + h23;
  }
  for (; i < n; i++) sum += a[i] * b[i];
  return sum;
}

// MatVecMul (TensorOps.cs:63-72): result[r] = Dot(mat[r, :], vec).
OR_API void or_matvec_f32(const float* mat, const float* vec, float* res, int64_t rows,
                          int cols, int nthreads) {
#pragma omp parallel for schedule(static) num_threads(nthreads > 0 ? nthreads : 1)
  for (int64_t r = 0; r < rows; r++) res[r] = or_dot(mat + r * (int64_t)cols, vec, cols);
}

// The reference dequantises every weight to f32 at load time
// (DequantizeTensor, Quantization.cs:415-469) and then runs MatVecMul over the
// f32 copy.  This does the same arithmetic one row at a time (identical
// values, bounded memory): y[b][r] = Dot(dequant(W[r, :]), x[b]).
OR_API int or_qmatvec(int qt, const uint8_t* w, int64_t rows, int cols, const float* x,
                      float* y, int batch, int nthreads) {
  int bs = or_block_size(qt), bb = or_block_bytes(qt);
  if (qt != QT_F32 && (bs <= 1 || cols % bs)) return -1;
  int64_t row_bytes = qt == QT_F32 ? (int64_t)cols * 4 : (int64_t)(cols / bs) * bb;
  int bad = 0;
#pragma omp parallel num_threads(nthreads > 0 ? nthreads : 1)
  {
    std::vector<float> row((size_t)cols);
#pragma omp for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
      if (or_dequant_tensor(qt, w + r * row_bytes, cols, row.data())) bad = 1;
      for (int b = 0; b < batch; b++)
        y[(int64_t)b * rows + r] = or_dot(row.data(), x + (int64_t)b * cols, cols);
    }
  }
  return bad ? -1 : 0;
}

// MatMul (TensorOps.cs:79-112): 32-tiled, c cleared then c += a*b with the
// k loop innermost-but-one.  For every (i, j) the k terms are added in
// ascending order, each product rounded before the add.
OR_API void or_matmul(const float* a, const float* b, float* c, int M, int K, int N) {
  const int T = 32;
  memset(c, 0, sizeof(float) * (size_t)M * N);
  for (int i = 0; i < M; i += T)
    for (int j = 0; j < N; j += T)
      for (int k = 0; k < K; k += T) {
        int iEnd = std::min(i + T, M), jEnd = std::min(j + T, N), kEnd = std::min(k + T, K);
        for (int ii = i; ii < iEnd; ii++)
          for (int kk = k; kk < kEnd; kk++) {
            float aVal = a[(int64_t)ii * K + kk];
            for (int jj = j; jj < jEnd; jj++) {
              float p = aVal * b[(int64_t)kk * N + jj];
              c[(int64_t)ii * N + jj] = c[(int64_t)ii * N + jj] + p;
            }
          }
      }
}

// Softmax (TensorOps.cs:115-132).
OR_API void or_softmax(float* x, int n) {
  float mx = -3.40282347e+38f;  // float.MinValue
  for (int i = 0; i < n; i++)
    if (x[i] > mx) mx = x[i];
  float sum = 0.0f;
  for (int i = 0; i < n; i++) {
    x[i] = expf(x[i] - mx);
    sum += x[i];
  }
  float inv = 1.0f / sum;
  for (int i = 0; i < n; i++) x[i] *= inv;
}

// RmsNorm (TensorOps.cs:135-145): scale = 1 / sqrt(sumSq / n + eps);
// out = (x * scale) * w.
OR_API void or_rmsnorm(float* out, const float* x, const float* w, int n, float eps) {
  float ss = 0.0f;
  for (int i = 0; i < n; i++) ss += x[i] * x[i];
  float scale = 1.0f / sqrtf(ss / (float)n + eps);
  for (int i = 0; i < n; i++) out[i] = x[i] * scale * w[i];
}

// AddInPlace (:149-165), MulInPlace (:169-185), SiLU (:191-195),
// AddScaled (:211-215).
OR_API void or_add_inplace(float* a, const float* b, int n) {
  for (int i = 0; i < n; i++) a[i] = a[i] + b[i];
}
OR_API void or_mul_inplace(float* a, const float* b, int n) {
  for (int i = 0; i < n; i++) a[i] = a[i] * b[i];
}
OR_API void or_silu(float* x, int n) {
  for (int i = 0; i < n; i++) x[i] = x[i] / (1.0f + expf(-x[i]));
}
OR_API void or_add_scaled(float* dst, const float* src, float s, int n) {
  for (int i = 0; i < n; i++) dst[i] += src[i] * s;
}

// ArgMax (TensorOps.cs:221-234; SamplingPipeline.cs:83-89): first index of
// the maximum under strict '>'.
OR_API int or_argmax(const float* x, int64_t n) {
  int64_t best = 0;
  float bv = x[0];
  for (int64_t i = 1; i < n; i++)
    if (x[i] > bv) { bv = x[i]; best = i; }
  return (int)best;
}

// ---------------------------------------------------------------------------
// RotaryEmbedding.cs
// ---------------------------------------------------------------------------

// ApplyToHead (RotaryEmbedding.cs:42-61): adjacent pairs (i, i+1),
// freq = 1 / powf(theta, i / headDim), angle = position * freq.
static void rope_head(float* head, int position, int hd, float theta) {
  for (int i = 0; i < hd; i += 2) {
    float freq = 1.0f / powf(theta, (float)i / (float)hd);
    float angle = (float)position * freq;
    float c = cosf(angle), s = sinf(angle);
    float x0 = head[i], x1 = head[i + 1];
    head[i] = x0 * c - x1 * s;
    head[i + 1] = x0 * s + x1 * c;
  }
}

// Apply (RotaryEmbedding.cs:24-40).
OR_API void or_rope_apply(float* q, float* k, int position, int hd, int nh, int nkv,
                          float theta) {
  for (int h = 0; h < nh; h++) rope_head(q + h * hd, position, hd, theta);
  for (int h = 0; h < nkv; h++) rope_head(k + h * hd, position, hd, theta);
}

// cos/sin table with exactly the angles ApplyToHead forms:
// tab[(pos * hd/2 + i/2) * 2 + {0,1}] = {cos, sin}.
OR_API void or_rope_table(float* tab, int npos, int hd, float theta) {
  for (int p = 0; p < npos; p++)
    for (int i = 0; i < hd; i += 2) {
      float freq = 1.0f / powf(theta, (float)i / (float)hd);
      float angle = (float)p * freq;
      tab[((int64_t)p * (hd / 2) + i / 2) * 2 + 0] = cosf(angle);
      tab[((int64_t)p * (hd / 2) + i / 2) * 2 + 1] = sinf(angle);
    }
}

// ---------------------------------------------------------------------------
// Attention inside Transformer.Forward (Transformer.cs:99-129)
// ---------------------------------------------------------------------------

// K/V are [kv_len][nkv][hd] (KVCache.cs:60-71 index pos*nKv*hd + kvh*hd).
// out[h*hd + d] = sum_t softmax_t(Dot(q_h, K_t) * (1/sqrt(hd))) * V_t[d],
// accumulated with AddScaled in ascending t.
OR_API void or_attention_decode(const float* q, const float* K, const float* V, int kv_len,
                                int nh, int nkv, int hd, float* out, int nthreads) {
  int groups = nh / nkv;
  float scale = 1.0f / sqrtf((float)hd);
#pragma omp parallel num_threads(nthreads > 0 ? nthreads : 1)
  {
    std::vector<float> scores((size_t)kv_len);
#pragma omp for schedule(static)
    for (int h = 0; h < nh; h++) {
      int kvh = h / groups;
      const float* qh = q + (int64_t)h * hd;
      for (int t = 0; t < kv_len; t++)
        scores[t] = or_dot(qh, K + ((int64_t)t * nkv + kvh) * hd, hd) * scale;
      or_softmax(scores.data(), kv_len);
      float* oh = out + (int64_t)h * hd;
      for (int d = 0; d < hd; d++) oh[d] = 0.0f;
      for (int t = 0; t < kv_len; t++)
        or_add_scaled(oh, V + ((int64_t)t * nkv + kvh) * hd, scores[t], hd);
    }
  }
}

// ---------------------------------------------------------------------------
// FlashAttention.cs (prefill attention semantics)
// ---------------------------------------------------------------------------

// SimdDot (FlashAttention.cs:328-348): 8 lanes, lanes summed 0..7 in order.
static float fa_simd_dot(const float* a, const float* b, int len) {
  float v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  int d = 0;
  for (; d + 8 <= len; d += 8)
    for (int j = 0; j < 8; j++) {
      float p = a[d + j] * b[d + j];
      v[j] = v[j] + p;
    }
  float r = 0.0f;
  for (int j = 0; j < 8; j++) r += v[j];
  for (; d < len; d++) r += a[d] * b[d];
  return r;
}

// Forward (FlashAttention.cs:59-167) for one head: Q [seq][hd], K/V [kv][hd].
OR_API void or_flash_attention(const float* Q, const float* K, const float* V, float* out,
                               int seq, int kv, int hd, float scale, int causal,
                               int start_pos) {
  const int BQ = 64, BKV = 64;  // BLOCK_SIZE_Q / BLOCK_SIZE_KV (:38-39)
  int blockQ = std::min(BQ, seq), blockKV = std::min(BKV, kv);
  std::vector<float> rowMax(blockQ), rowSum(blockQ), rowOut((size_t)blockQ * hd),
      s((size_t)blockQ * blockKV);
  const float NEG_INF = -INFINITY;
  for (int qi = 0; qi < seq; qi += blockQ) {
    int qBlock = std::min(qi + blockQ, seq) - qi;
    for (int r = 0; r < qBlock; r++) { rowMax[r] = NEG_INF; rowSum[r] = 0.0f; }
    std::fill(rowOut.begin(), rowOut.begin() + (size_t)qBlock * hd, 0.0f);
    for (int ki = 0; ki < kv; ki += blockKV) {
      int kBlock = std::min(ki + blockKV, kv) - ki;
      // ComputeAttentionScores (:173-203)
      for (int a = 0; a < qBlock; a++)
        for (int b = 0; b < kBlock; b++)
          s[a * kBlock + b] =
              fa_simd_dot(Q + (int64_t)(qi + a) * hd, K + (int64_t)(ki + b) * hd, hd) * scale;
      // ApplyCausalMask (:206-224)
      if (causal)
        for (int a = 0; a < qBlock; a++) {
          int qpos = start_pos + qi + a;
          for (int b = 0; b < kBlock; b++)
            if (ki + b > qpos) s[a * kBlock + b] = NEG_INF;
        }
      // UpdateOnlineSoftmax (:238-325)
      for (int a = 0; a < qBlock; a++) {
        float bmax = NEG_INF;
        for (int b = 0; b < kBlock; b++)
          if (s[a * kBlock + b] > bmax) bmax = s[a * kBlock + b];
        if (isinf(bmax) && bmax < 0) continue;
        float oldMax = rowMax[a];
        float newMax = std::max(oldMax, bmax);
        float rescale = (isinf(oldMax) && oldMax < 0) ? 0.0f : expf(oldMax - newMax);
        rowSum[a] *= rescale;
        float* o = rowOut.data() + (size_t)a * hd;
        if (rescale != 0.0f && rescale != 1.0f)
          for (int d = 0; d < hd; d++) o[d] *= rescale;
        for (int b = 0; b < kBlock; b++) {
          float sv = s[a * kBlock + b];
          if (isinf(sv) && sv < 0) continue;
          float p = expf(sv - newMax);
          rowSum[a] += p;
          const float* vr = V + (int64_t)(ki + b) * hd;
          for (int d = 0; d < hd; d++) {
            float t = p * vr[d];
            o[d] = o[d] + t;
          }
        }
        rowMax[a] = newMax;
      }
    }
    for (int r = 0; r < qBlock; r++) {
      float inv = rowSum[r] > 0 ? 1.0f / rowSum[r] : 0.0f;
      for (int d = 0; d < hd; d++)
        out[(int64_t)(qi + r) * hd + d] = rowOut[(size_t)r * hd + d] * inv;
    }
  }
}

// ---------------------------------------------------------------------------
// Transformer.Forward (Transformer.cs:67-162) over quantised weights
// ---------------------------------------------------------------------------

struct OrConfig {
  int n_layers, hidden, inter, n_heads, n_kv_heads, head_dim, vocab, max_seq;
  float eps, theta;
};

struct OrTensor {
  int qt;
  const uint8_t* data;  // row-major [rows][cols] in GGUF blocks (borrowed)
};

enum { W_Q, W_K, W_V, W_O, W_GATE, W_UP, W_DOWN, W_COUNT };

struct OrModel {
  OrConfig c;
  int n_seq;
  OrTensor emb, lm_head;
  std::vector<OrTensor> w;         // [layer * W_COUNT + which]
  std::vector<const float*> norms;  // [layer * 2 + {attn, ffn}], final at end
  const float* final_norm;
  std::vector<float> kcache, vcache;  // [seq][layer][max_seq][nkv*hd] f32
  int nthreads;
};

OR_API void* or_model_create(int n_layers, int hidden, int inter, int n_heads, int n_kv_heads,
                             int head_dim, int vocab, int max_seq, float eps, float theta,
                             int n_seq, int nthreads) {
  // The reference sizes its attention output buffer by HiddenSize
  // (Transformer.cs:50) and so needs HiddenSize == NumAttentionHeads * HeadDim;
  // it would throw on other shapes, the restatement refuses them.
  if (hidden != n_heads * head_dim) return nullptr;
  OrModel* m = new OrModel();
  m->c = {n_layers, hidden, inter, n_heads, n_kv_heads, head_dim, vocab, max_seq, eps, theta};
  m->n_seq = n_seq;
  m->w.assign((size_t)n_layers * W_COUNT, OrTensor{0, nullptr});
  m->norms.assign((size_t)n_layers * 2, nullptr);
  m->final_norm = nullptr;
  size_t per = (size_t)n_seq * n_layers * max_seq * n_kv_heads * head_dim;
  m->kcache.assign(per, 0.0f);
  m->vcache.assign(per, 0.0f);
  m->nthreads = nthreads;
  return m;
}

OR_API void or_model_free(void* p) { delete (OrModel*)p; }

// which: 0..6 = Wq, Wk, Wv, Wo, Wgate, Wup, Wdown; 7 = attn norm, 8 = ffn
// norm (f32, `data` is float*); layer -1: which 0 = token embedding,
// 1 = lm_head, 2 = final norm.
OR_API void or_model_set(void* p, int layer, int which, int qt, const void* data) {
  OrModel* m = (OrModel*)p;
  if (layer < 0) {
    if (which == 0) m->emb = {qt, (const uint8_t*)data};
    else if (which == 1) m->lm_head = {qt, (const uint8_t*)data};
    else m->final_norm = (const float*)data;
    return;
  }
  if (which < W_COUNT) m->w[(size_t)layer * W_COUNT + which] = {qt, (const uint8_t*)data};
  else m->norms[(size_t)layer * 2 + (which - W_COUNT)] = (const float*)data;
}

static inline float* kv_ptr(OrModel* m, std::vector<float>& cache, int seq, int layer, int pos) {
  size_t stride = (size_t)m->c.n_kv_heads * m->c.head_dim;
  return cache.data() + (((size_t)seq * m->c.n_layers + layer) * m->c.max_seq + pos) * stride;
}

// Fill cache positions [0, len) of (seq, layer) from f16 K/V [len][nkv*hd].
OR_API void or_model_kv_fill(void* p, int seq, int layer, const uint16_t* k, const uint16_t* v,
                             int len) {
  OrModel* m = (OrModel*)p;
  size_t n = (size_t)len * m->c.n_kv_heads * m->c.head_dim;
  float* kd = kv_ptr(m, m->kcache, seq, layer, 0);
  float* vd = kv_ptr(m, m->vcache, seq, layer, 0);
  for (size_t i = 0; i < n; i++) {
    kd[i] = or_half_to_float(k[i]);
    vd[i] = or_half_to_float(v[i]);
  }
}

static inline float round_f16(float x) {
  // binary32 -> binary16 (round to nearest even) -> binary32
  uint32_t u;
  memcpy(&u, &x, 4);
  uint32_t sign = u & 0x80000000u, ax = u & 0x7FFFFFFFu;
  if (ax >= 0x7F800000u) return x;
  float a = fabsf(x);
  if (a >= 65520.0f) return sign ? -INFINITY : INFINITY;
  int e;
  frexpf(a, &e);  // a = f * 2^e, f in [0.5, 1)
  int ulp_exp = std::max(e - 11, -24);
  float ulp = ldexpf(1.0f, ulp_exp);
  float r = nearbyintf(a / ulp) * ulp;  // exact scaling by a power of two; RNE
  return sign ? -r : r;
}

static void qmatvec_rows(OrModel* m, const OrTensor& t, int64_t rows, int cols, const float* x,
                         float* y) {
  or_qmatvec(t.qt, t.data, rows, cols, x, y, 1, m->nthreads);
}

// One decode step for sequence `seq` (Transformer.cs:67-162).  K/V written
// into the cache are rounded through binary16 when kv_round_f16 is set (the
// device cache is f16; the reference's is f32, KVCache.cs:15-16).
OR_API int or_model_forward(void* p, int seq, int token, int pos, int kv_round_f16,
                            float* logits) {
  OrModel* m = (OrModel*)p;
  const OrConfig& c = m->c;
  int h = c.hidden, hd = c.head_dim, nh = c.n_heads, nkv = c.n_kv_heads;
  if (pos >= c.max_seq) return -1;
  std::vector<float> x(h), xn(h), q((size_t)nh * hd), k((size_t)nkv * hd),
      v((size_t)nkv * hd), att(h), proj(h), gate(c.inter), up(c.inter), down(h);
  // Token embedding: row `token` of the dequantised table (:76).
  {
    int bs = or_block_size(m->emb.qt), bb = or_block_bytes(m->emb.qt);
    int64_t row_bytes = m->emb.qt == QT_F32 ? (int64_t)h * 4 : (int64_t)(h / bs) * bb;
    if (or_dequant_tensor(m->emb.qt, m->emb.data + (int64_t)token * row_bytes, h, x.data()))
      return -2;
  }
  for (int l = 0; l < c.n_layers; l++) {
    const OrTensor* w = &m->w[(size_t)l * W_COUNT];
    or_rmsnorm(xn.data(), x.data(), m->norms[(size_t)l * 2 + 0], h, c.eps);  // :86
    qmatvec_rows(m, w[W_Q], (int64_t)nh * hd, h, xn.data(), q.data());       // :89
    qmatvec_rows(m, w[W_K], (int64_t)nkv * hd, h, xn.data(), k.data());      // :90
    qmatvec_rows(m, w[W_V], (int64_t)nkv * hd, h, xn.data(), v.data());      // :91
    or_rope_apply(q.data(), k.data(), pos, hd, nh, nkv, c.theta);            // :94
    float* kc = kv_ptr(m, m->kcache, seq, l, pos);                          // :97
    float* vc = kv_ptr(m, m->vcache, seq, l, pos);
    for (int i = 0; i < nkv * hd; i++) {
      kc[i] = kv_round_f16 ? round_f16(k[i]) : k[i];
      vc[i] = kv_round_f16 ? round_f16(v[i]) : v[i];
    }
    or_attention_decode(q.data(), kv_ptr(m, m->kcache, seq, l, 0),
                        kv_ptr(m, m->vcache, seq, l, 0), pos + 1, nh, nkv, hd, att.data(),
                        m->nthreads);                                        // :99-129
    qmatvec_rows(m, w[W_O], h, h, att.data(), proj.data());                 // :132
    or_add_inplace(x.data(), proj.data(), h);                               // :135
    or_rmsnorm(xn.data(), x.data(), m->norms[(size_t)l * 2 + 1], h, c.eps); // :140
    qmatvec_rows(m, w[W_GATE], c.inter, h, xn.data(), gate.data());        // :143
    qmatvec_rows(m, w[W_UP], c.inter, h, xn.data(), up.data());            // :144
    or_silu(gate.data(), c.inter);                                          // :147
    or_mul_inplace(gate.data(), up.data(), c.inter);                        // :148
    qmatvec_rows(m, w[W_DOWN], h, c.inter, gate.data(), down.data());      // :151
    or_add_inplace(x.data(), down.data(), h);                               // :154
  }
  or_rmsnorm(xn.data(), x.data(), m->final_norm, h, c.eps);                 // :158
  qmatvec_rows(m, m->lm_head, c.vocab, h, xn.data(), logits);               // :159
  return 0;
}

// The cached K and V of positions [0, len) of (seq, layer) in the reference
// layout [pos][kv head][dim] (KVCache.GetKey / GetValue, KVCache.cs:60-71).
OR_API void or_model_kv_get(void* p, int seq, int layer, int len, float* k, float* v) {
  OrModel* m = (OrModel*)p;
  const size_t n = (size_t)len * m->c.n_kv_heads * m->c.head_dim;
  memcpy(k, kv_ptr(m, m->kcache, seq, layer, 0), n * sizeof(float));
  memcpy(v, kv_ptr(m, m->vcache, seq, layer, 0), n * sizeof(float));
}

// binary32 -> binary16 -> binary32 helper exported for tests.
OR_API float or_round_f16(float x) { return round_f16(x); }

OR_API int or_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
