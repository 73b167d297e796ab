// The f32 C ABI that SharpInfer's CudaBackend and FlashAttention bind
// (library `sharpinfer_cuda`: src/SharpInfer.Gpu/CudaBackend.cs:141-163,
// src/SharpInfer.Core/Layers/FlashAttention.cs:380-384,
// src/SharpInfer.Core/Tensors/HardwareBackends.cs:438-442), implemented on the
// B200 so that the existing managed backend runs unchanged.
//
// Conventions of that interface: void returns (failures are recorded for
// si_last_error() and otherwise ignored, as the reference does), a handle per
// backend instance (here an si_ctx*), and pointers that are host memory
// pinned only for the call -- each call copies its inputs to the device,
// computes on the context stream, copies the result back and synchronises.
// Device pointers (cudaMalloc'd) are accepted too and used in place.
//
// Semantics are those of the managed CPU operators in TensorOps.cs: MatVecMul
// :63-72, MatMul :79-112, Softmax :115-132, RmsNorm :135-145, AddInPlace
// :149-165, SiLU :191-195; flash_attention_forward follows
// FlashAttention.Forward :59-167 with the causal offset startPos = kvLen -
// seqLen (the queries are the last seqLen positions).
#include <math.h>
#include <string.h>

#include "common.cuh"

namespace si {
namespace {

__global__ void __launch_bounds__(256) k_matvec_f32(const float* __restrict__ A, const float* __restrict__ x,
                                                    float* __restrict__ y, int64_t rows, int cols) {
  const int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const float* a = A + r * cols;
  float s = 0.f;
  if ((cols & 3) == 0 && (((uintptr_t)a | (uintptr_t)x) & 15) == 0) {
    for (int c = lane * 4; c < cols; c += 128) {
      const float4 av = __ldg((const float4*)(a + c)), xv = __ldg((const float4*)(x + c));
      s = fmaf(av.x, xv.x, s);
      s = fmaf(av.y, xv.y, s);
      s = fmaf(av.z, xv.z, s);
      s = fmaf(av.w, xv.w, s);
    }
  } else {
    for (int c = lane; c < cols; c += 32) s = fmaf(__ldg(a + c), __ldg(x + c), s);
  }
  s = warp_sum(s);
  if (lane == 0) y[r] = s;
}

// C[M][N] = A[M][K] * B[K][N], row-major f32: 64 x 64 tiles, 4 x 4 per thread.
__global__ void __launch_bounds__(256) k_matmul_f32(const float* __restrict__ A, const float* __restrict__ B,
                                                    float* __restrict__ C, int M, int K, int N) {
  __shared__ float As[16][64 + 4];
  __shared__ float Bs[16][64 + 4];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += 16) {
    for (int i = threadIdx.x; i < 64 * 16; i += 256) {
      const int r = i >> 4, c = i & 15;  // A tile: 64 rows x 16 k
      const int gm = m0 + r, gk = k0 + c;
      As[c][r] = (gm < M && gk < K) ? A[(int64_t)gm * K + gk] : 0.f;
      const int kr = i >> 6, nc = i & 63;  // B tile: 16 k x 64 cols
      const int bk = k0 + kr, bn = n0 + nc;
      Bs[kr][nc] = (bk < K && bn < N) ? B[(int64_t)bk * N + bn] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; kk++) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; i++) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; j++) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int gm = m0 + ty * 4 + i;
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int gn = n0 + tx * 4 + j;
      if (gn < N) C[(int64_t)gm * N + gn] = acc[i][j];
    }
  }
}

__device__ float block_reduce(float v, bool is_max, float* red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = is_max ? warp_max(v) : warp_sum(v);
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float t = is_max ? -INFINITY : 0.f;
  for (int i = 0; i < nw; i++) t = is_max ? fmaxf(t, red[i]) : t + red[i];
  return t;
}

// Softmax in place, one CTA: max (float.MinValue start), exp(x - max), sum, * (1 / sum).
__global__ void __launch_bounds__(1024) k_softmax(float* __restrict__ x, int n) {
  __shared__ float red[32];
  float m = -3.40282347e+38f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, x[i]);
  m = block_reduce(m, true, red);
  float s = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float e = expf(x[i] - m);
    x[i] = e;
    s += e;
  }
  s = block_reduce(s, false, red);
  const float inv = 1.0f / s;
  for (int i = threadIdx.x; i < n; i += blockDim.x) x[i] *= inv;
}

// out = (x * (1 / sqrt(sum(x^2) / n + eps))) * w, one CTA.
__global__ void __launch_bounds__(1024) k_rmsnorm(float* __restrict__ out, const float* __restrict__ x,
                                                  const float* __restrict__ w, int n, float eps) {
  __shared__ float red[32];
  float ss = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) ss = __fadd_rn(ss, __fmul_rn(x[i], x[i]));
  ss = block_reduce(ss, false, red);
  const float scale = 1.0f / sqrtf(ss / (float)n + eps);
  for (int i = threadIdx.x; i < n; i += blockDim.x) out[i] = __fmul_rn(__fmul_rn(x[i], scale), w[i]);
}

__global__ void k_silu(float* __restrict__ x, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) x[i] = __fdiv_rn(x[i], __fadd_rn(1.0f, expf(-x[i])));
}

__global__ void k_add(float* __restrict__ a, const float* __restrict__ b, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) a[i] = __fadd_rn(a[i], b[i]);
}

// f32 attention, one warp per query row: scores over the unmasked keys with
// an online softmax, lane l holding dims l, l+32, ... (head_dim <= 256).
// Q, O: [B][H][S][D]; K, V: [B][H][KV][D].  Query i sees keys j <= i + (KV - S);
// a row with no visible key is 0 (FlashAttention.cs:155-163).
__global__ void __launch_bounds__(256) k_attn_f32(const float* __restrict__ Q, const float* __restrict__ K,
                                                  const float* __restrict__ V, float* __restrict__ O, int64_t nrows,
                                                  int S, int KV, int D, float scale, int causal) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);  // (b*H + h)*S + i
  if (row >= nrows) return;
  const int64_t bh = row / S;
  const int i = (int)(row % S);
  const float* q = Q + row * D;
  const float* kb = K + bh * KV * D;
  const float* vb = V + bh * KV * D;
  float qv[8], o[8];
  const int nd = (D + 31) / 32;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const int d = lane + 32 * j;
    qv[j] = (j < nd && d < D) ? q[d] : 0.f;
    o[j] = 0.f;
  }
  const int last = causal ? min(KV - 1, i + (KV - S)) : KV - 1;
  float m = -INFINITY, l = 0.f;
  for (int t = 0; t <= last; t++) {
    const float* kr = kb + (int64_t)t * D;
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const int d = lane + 32 * j;
      if (j < nd && d < D) s = fmaf(qv[j], __ldg(kr + d), s);
    }
    s = warp_sum(s) * scale;
    const float mn = fmaxf(m, s);
    const float r = m == -INFINITY ? 0.f : expf(m - mn);
    const float p = expf(s - mn);
    l = l * r + p;
    const float* vr = vb + (int64_t)t * D;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const int d = lane + 32 * j;
      if (j < nd && d < D) o[j] = fmaf(p, __ldg(vr + d), o[j] * r);
    }
    m = mn;
  }
  const float inv = l > 0.f ? 1.0f / l : 0.f;
  float* out = O + row * D;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const int d = lane + 32 * j;
    if (j < nd && d < D) out[d] = o[j] * inv;
  }
}

bool is_device(const void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

// A host or device buffer seen from the device: host buffers are staged.
struct Arg {
  const void* user;
  size_t bytes;
  bool dev;
  void* d;
};

int stage_in(si_ctx* c, Arg& a, int slot, bool copy) {
  a.dev = is_device(a.user);
  if (a.dev) {
    a.d = const_cast<void*>(a.user);
    return SI_OK;
  }
  SI_TRY(ensure(c->stage[slot], a.bytes));
  a.d = c->stage[slot].ptr;
  if (copy) SI_CUDA(cudaMemcpyAsync(a.d, a.user, a.bytes, cudaMemcpyHostToDevice, c->stream));
  return SI_OK;
}

int stage_out(si_ctx* c, const Arg& a) {
  if (!a.dev) SI_CUDA(cudaMemcpyAsync(const_cast<void*>(a.user), a.d, a.bytes, cudaMemcpyDeviceToHost, c->stream));
  SI_CUDA(cudaStreamSynchronize(c->stream));
  return SI_OK;
}

int matvec(si_ctx* c, const float* mat, const float* vec, float* res, int rows, int cols) {
  if (!c || !mat || !vec || !res || rows < 0 || cols < 0) SI_FAIL(SI_ERR_INVALID, "cuda_mat_vec_mul: bad arguments");
  if (rows == 0) return SI_OK;
  SI_TRY(bind_device(c));
  Arg A{mat, (size_t)rows * cols * 4}, X{vec, (size_t)cols * 4}, Y{res, (size_t)rows * 4};
  SI_TRY(stage_in(c, A, 0, true));
  SI_TRY(stage_in(c, X, 1, true));
  SI_TRY(stage_in(c, Y, 2, false));
  k_matvec_f32<<<(unsigned)((rows + 7) / 8), 256, 0, c->stream>>>((const float*)A.d, (const float*)X.d, (float*)Y.d,
                                                                 rows, cols);
  SI_CUDA(cudaGetLastError());
  return stage_out(c, Y);
}

int matmul(si_ctx* c, const float* a, const float* b, float* out, int M, int K, int N) {
  if (!c || !a || !b || !out || M < 0 || K < 0 || N < 0) SI_FAIL(SI_ERR_INVALID, "cuda_mat_mul: bad arguments");
  if (M == 0 || N == 0) return SI_OK;
  SI_TRY(bind_device(c));
  Arg A{a, (size_t)M * K * 4}, B{b, (size_t)K * N * 4}, C{out, (size_t)M * N * 4};
  SI_TRY(stage_in(c, A, 0, true));
  SI_TRY(stage_in(c, B, 1, true));
  SI_TRY(stage_in(c, C, 2, false));
  dim3 grid((unsigned)((N + 63) / 64), (unsigned)((M + 63) / 64));
  k_matmul_f32<<<grid, 256, 0, c->stream>>>((const float*)A.d, (const float*)B.d, (float*)C.d, M, K, N);
  SI_CUDA(cudaGetLastError());
  return stage_out(c, C);
}

int elementwise(si_ctx* c, const char* what, float* x, const float* y, const float* w, float* out, int n,
                float eps) {
  if (!c || !x || n < 0) SI_FAIL(SI_ERR_INVALID, "%s: bad arguments", what);
  if (n == 0) return SI_OK;
  SI_TRY(bind_device(c));
  const size_t bytes = (size_t)n * 4;
  Arg X{x, bytes};
  SI_TRY(stage_in(c, X, 0, true));
  if (!strcmp(what, "cuda_softmax")) {
    k_softmax<<<1, 1024, 0, c->stream>>>((float*)X.d, n);
    SI_CUDA(cudaGetLastError());
    return stage_out(c, X);
  }
  if (!strcmp(what, "cuda_silu")) {
    k_silu<<<(unsigned)((n + 255) / 256), 256, 0, c->stream>>>((float*)X.d, n);
    SI_CUDA(cudaGetLastError());
    return stage_out(c, X);
  }
  if (!strcmp(what, "cuda_add_inplace")) {
    if (!y) SI_FAIL(SI_ERR_INVALID, "cuda_add_inplace: NULL b");
    Arg Yb{y, bytes};
    SI_TRY(stage_in(c, Yb, 1, true));
    k_add<<<(unsigned)((n + 255) / 256), 256, 0, c->stream>>>((float*)X.d, (const float*)Yb.d, n);
    SI_CUDA(cudaGetLastError());
    return stage_out(c, X);
  }
  // cuda_rms_norm: x is the input, out the output
  if (!w || !out) SI_FAIL(SI_ERR_INVALID, "cuda_rms_norm: NULL argument");
  Arg W{w, bytes}, Out{out, bytes};
  SI_TRY(stage_in(c, W, 1, true));
  SI_TRY(stage_in(c, Out, 2, false));
  k_rmsnorm<<<1, 1024, 0, c->stream>>>((float*)Out.d, (const float*)X.d, (const float*)W.d, n, eps);
  SI_CUDA(cudaGetLastError());
  return stage_out(c, Out);
}

}  // namespace
}  // namespace si

using namespace si;

extern "C" {

SI_EXPORT void* cuda_init(int device) {
  si_ctx* c = nullptr;
  if (si_init(device, &c) != SI_OK) return nullptr;
  return c;
}

SI_EXPORT void cuda_cleanup(void* handle) { si_shutdown((si_ctx*)handle); }

SI_EXPORT void cuda_device_name(void* handle, char* buf, int len) {
  if (si_device_name((si_ctx*)handle, buf, len) != SI_OK && buf && len > 0) buf[0] = 0;
}

SI_EXPORT int cuda_is_available(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n > 0 ? 1 : 0;
}

SI_EXPORT const char* cuda_device_name_str(void) {
  static thread_local char name[256];
  cudaDeviceProp p;
  if (cudaGetDeviceProperties(&p, 0) != cudaSuccess) {
    cudaGetLastError();
    strcpy(name, "none");
  } else {
    strncpy(name, p.name, sizeof(name) - 1);
    name[sizeof(name) - 1] = 0;
  }
  return name;
}

SI_EXPORT void cuda_mat_vec_mul(void* h, const float* mat, const float* vec, float* res, int rows, int cols) {
  clear_error();
  matvec((si_ctx*)h, mat, vec, res, rows, cols);
}

SI_EXPORT void cuda_mat_mul(void* h, const float* a, const float* b, float* c, int M, int K, int N) {
  clear_error();
  matmul((si_ctx*)h, a, b, c, M, K, N);
}

SI_EXPORT void cuda_softmax(void* h, float* x, int len) {
  clear_error();
  elementwise((si_ctx*)h, "cuda_softmax", x, nullptr, nullptr, nullptr, len, 0.f);
}

SI_EXPORT void cuda_rms_norm(void* h, float* output, const float* x, const float* weight, int size, float eps) {
  clear_error();
  elementwise((si_ctx*)h, "cuda_rms_norm", const_cast<float*>(x), nullptr, weight, output, size, eps);
}

SI_EXPORT void cuda_silu(void* h, float* x, int len) {
  clear_error();
  elementwise((si_ctx*)h, "cuda_silu", x, nullptr, nullptr, nullptr, len, 0.f);
}

SI_EXPORT void cuda_add_inplace(void* h, float* a, const float* b, int len) {
  clear_error();
  elementwise((si_ctx*)h, "cuda_add_inplace", a, b, nullptr, nullptr, len, 0.f);
}

// No context in this signature: a per-thread context on the current device
// holds the staging buffers.
SI_EXPORT void flash_attention_forward(void* Q, void* K, void* V, void* O, int batch, int heads, int seq, int kv,
                                       int head_dim, float scale, int causal) {
  clear_error();
  static thread_local si_ctx* ctx = nullptr;
  static thread_local int ctx_dev = -1;
  auto run = [&]() -> int {
    if (!Q || !K || !V || !O || batch < 0 || heads < 0 || seq < 0 || kv < 0 || head_dim <= 0 || head_dim > 256)
      SI_FAIL(SI_ERR_INVALID, "flash_attention_forward: bad arguments (head_dim 1..256)");
    if (batch == 0 || heads == 0 || seq == 0) return SI_OK;
    int dev = 0;
    SI_CUDA(cudaGetDevice(&dev));
    if (!ctx || ctx_dev != dev) {
      if (ctx) si_shutdown(ctx);
      ctx = nullptr;
      SI_TRY(si_init(dev, &ctx));
      ctx_dev = dev;
    }
    const size_t qb = (size_t)batch * heads * seq * head_dim * 4, kb = (size_t)batch * heads * kv * head_dim * 4;
    Arg q{Q, qb}, k{K, kb}, v{V, kb}, o{O, qb};
    SI_TRY(stage_in(ctx, q, 0, true));
    SI_TRY(stage_in(ctx, k, 1, true));
    SI_TRY(stage_in(ctx, v, 2, true));
    SI_TRY(stage_in(ctx, o, 3, false));
    const int64_t rows = (int64_t)batch * heads * seq;
    k_attn_f32<<<(unsigned)((rows + 7) / 8), 256, 0, ctx->stream>>>(
        (const float*)q.d, (const float*)k.d, (const float*)v.d, (float*)o.d, rows, seq, kv, head_dim, scale, causal);
    SI_CUDA(cudaGetLastError());
    return stage_out(ctx, o);
  };
  run();
}

}  // extern "C"
