"""The f32 interface of SharpInfer's CudaBackend (cuda_* and
flash_attention_forward, src/SharpInfer.Gpu/CudaBackend.cs:141-163,
src/SharpInfer.Core/Layers/FlashAttention.cs:380-384) against the oracle's
TensorOps / FlashAttention restatements, called through the C ABI with host
buffers as the managed backend passes them."""
import ctypes

import numpy as np
import pytest

import oracle
from conftest import rel_l2
from sharpinfer_b200 import native as N

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def handle():
    L = N.load()
    h = L.cuda_init(0)
    assert h
    yield h
    L.cuda_cleanup(h)


def P(a):
    return a.ctypes.data


def test_probe_and_name(handle):
    L = N.load()
    assert L.cuda_is_available() == 1
    assert b"B200" in L.cuda_device_name_str()
    buf = ctypes.create_string_buffer(256)
    L.cuda_device_name(handle, buf, 256)
    assert b"B200" in buf.value


@pytest.mark.parametrize("rows,cols", [(1, 1), (7, 33), (1000, 4096), (4096, 14336), (3, 1)])
def test_mat_vec_mul(handle, rows, cols):
    rng = np.random.default_rng(rows * 7 + cols)
    A = rng.standard_normal((rows, cols)).astype(np.float32)
    x = rng.standard_normal(cols).astype(np.float32)
    y = np.full(rows, np.nan, np.float32)
    N.load().cuda_mat_vec_mul(handle, P(A), P(x), P(y), rows, cols)
    assert rel_l2(y, oracle.matvec_f32(A, x)) < 1e-5


@pytest.mark.parametrize("M,K,N_", [(1, 1, 1), (17, 33, 65), (64, 4096, 64), (130, 256, 70), (2, 5, 300)])
def test_mat_mul(handle, M, K, N_):
    rng = np.random.default_rng(M + K + N_)
    a = rng.standard_normal((M, K)).astype(np.float32)
    b = rng.standard_normal((K, N_)).astype(np.float32)
    c = np.full((M, N_), np.nan, np.float32)
    N.load().cuda_mat_mul(handle, P(a), P(b), P(c), M, K, N_)
    assert rel_l2(c, oracle.matmul(a, b)) < 1e-5


@pytest.mark.parametrize("n", [1, 33, 1000, 128256])
def test_softmax(handle, n):
    x = (np.random.default_rng(n).standard_normal(n) * 4).astype(np.float32)
    ref = oracle.softmax(x)
    N.load().cuda_softmax(handle, P(x), n)
    # the reference adds the n exponentials one after another in f32; at
    # n = 128256 that sum carries ~1e-4 relative rounding, which the device's
    # tree sum does not share -- hence the 1e-3 floating-point bar
    assert rel_l2(x, ref) < (1e-6 if n <= 1000 else 1e-3) and abs(float(x.sum()) - 1.0) < 1e-4


@pytest.mark.parametrize("n", [1, 4096, 14336])
def test_rms_norm(handle, n):
    rng = np.random.default_rng(n + 1)
    x = rng.standard_normal(n).astype(np.float32)
    w = (1 + 0.01 * rng.standard_normal(n)).astype(np.float32)
    out = np.full(n, np.nan, np.float32)
    N.load().cuda_rms_norm(handle, P(out), P(x), P(w), n, 1e-5)
    assert rel_l2(out, oracle.rmsnorm(x, w, 1e-5)) < 1e-6


@pytest.mark.parametrize("n", [1, 255, 14336])
def test_silu_and_add(handle, n):
    rng = np.random.default_rng(n + 2)
    x = (rng.standard_normal(n) * 3).astype(np.float32)
    ref = oracle.silu(x)
    N.load().cuda_silu(handle, P(x), n)
    assert rel_l2(x, ref) < 1e-6
    a = rng.standard_normal(n).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    want = a + b
    N.load().cuda_add_inplace(handle, P(a), P(b), n)
    assert np.array_equal(a, want)


def flash_ref(Q, K, V, scale, causal):
    B, H, S, D = Q.shape
    kv = K.shape[2]
    out = np.empty_like(Q)
    for b in range(B):
        for h in range(H):
            out[b, h] = oracle.flash_attention(Q[b, h], K[b, h], V[b, h], scale, causal, start_pos=kv - S)
    return out


@pytest.mark.parametrize("B,H,S,KV,D,causal", [(2, 3, 70, 130, 128, 1), (1, 2, 64, 64, 128, 1),
                                               (1, 1, 33, 200, 64, 0), (1, 2, 5, 3, 32, 1)])
def test_flash_attention_forward(B, H, S, KV, D, causal):
    rng = np.random.default_rng(S * KV + D)
    Q = rng.standard_normal((B, H, S, D)).astype(np.float32)
    K = rng.standard_normal((B, H, KV, D)).astype(np.float32)
    V = rng.standard_normal((B, H, KV, D)).astype(np.float32)
    O = np.full_like(Q, np.nan)
    scale = 1.0 / np.sqrt(D)
    N.load().flash_attention_forward(P(Q), P(K), P(V), P(O), B, H, S, KV, D, scale, causal)
    assert rel_l2(O, flash_ref(Q, K, V, scale, causal)) < 1e-5


def test_flash_attention_device_pointers():
    import torch
    rng = np.random.default_rng(5)
    Q = rng.standard_normal((1, 2, 40, 128)).astype(np.float32)
    K = rng.standard_normal((1, 2, 90, 128)).astype(np.float32)
    V = rng.standard_normal((1, 2, 90, 128)).astype(np.float32)
    tq, tk, tv = (torch.from_numpy(a).cuda() for a in (Q, K, V))
    to = torch.empty_like(tq)
    torch.cuda.synchronize()
    N.load().flash_attention_forward(tq.data_ptr(), tk.data_ptr(), tv.data_ptr(), to.data_ptr(), 1, 2, 40, 90, 128,
                                     0.125, 1)
    assert rel_l2(to.cpu().numpy(), flash_ref(Q, K, V, 0.125, 1)) < 1e-5


def test_bad_arguments_record_an_error(handle):
    L = N.load()
    x = np.zeros(4, np.float32)
    L.cuda_mat_vec_mul(handle, None, P(x), P(x), 2, 2)
    assert L.si_last_error()
    L.cuda_softmax(None, P(x), 4)  # no context: nothing happens, no crash
    assert L.si_last_error()
