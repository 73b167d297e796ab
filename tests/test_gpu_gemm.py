"""Prefill GEMM (si_qgemm, tcgen05) against the oracle: y = x W^T with W the
reference's dequantised weight (DequantizeTensor, Quantization.cs:415-469)
and the rows of x multiplied as TensorOps.MatMul / MatVecMul do
(TensorOps.cs:63-112).  x is bf16, so the oracle receives the same bf16
values as f32.  Bar: relative L2 1e-3 (measured ~1e-4: W is rounded to f16)."""
import numpy as np
import pytest

import oracle
from conftest import rel_l2
from sharpinfer_b200 import native as N
from sharpinfer_b200.backend import synth_blocks_host

pytestmark = pytest.mark.gpu
TOL = 1e-3


def bf16_round(a):
    b = np.ascontiguousarray(a, np.float32).view(np.uint32)
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    return r, (r.astype(np.uint32) << 16).view(np.float32)


@pytest.mark.parametrize("qt,M,rows,cols", [
    (N.SI_Q4_K, 128, 256, 256),     # one tile
    (N.SI_Q4_K, 300, 1000, 512),    # ragged M and N
    (N.SI_Q4_K, 1, 256, 4096),      # M = 1
    (N.SI_Q4_K, 512, 4096, 4096),   # Llama-3-8B q/o projection at M = 512
    (N.SI_Q6_K, 200, 520, 1024),
    (N.SI_Q8_0, 130, 384, 320),     # Q8_0, K not a multiple of 256
    (N.SI_Q4_K, 256, 512, 14336),   # down-projection K
    (N.SI_Q4_K, 1280, 4096, 256),   # enough 256-wide tiles for every SM: the 256-column variant
])
def test_qgemm_matches_oracle(ctx, qt, M, rows, cols):
    import torch
    blocks = synth_blocks_host(qt, rows, cols, 99, 5, N.SYNTH_PLAIN, 0.01)
    xb, xf = bf16_round(np.random.default_rng(M + rows).standard_normal((M, cols)))
    ref = oracle.qmatvec(qt, blocks, rows, cols, xf)
    w = ctx.upload(qt, blocks, rows, cols)
    y = ctx.qgemm(w, torch.from_numpy(xb.view(np.int16)).cuda().view(torch.bfloat16))
    ctx.synchronize()
    err = rel_l2(y.cpu().numpy(), ref)
    assert err < TOL, err
    w.free()


def test_qgemm_repeatable_and_rejects_bad_shapes(ctx):
    import torch
    blocks = synth_blocks_host(N.SI_Q4_K, 256, 512, 3, 1, N.SYNTH_PLAIN, 0.01)
    w = ctx.upload(N.SI_Q4_K, blocks, 256, 512)
    x = torch.randn(130, 512, device="cuda").to(torch.bfloat16)
    a = ctx.qgemm(w, x)
    b = ctx.qgemm(w, x)
    ctx.synchronize()
    assert torch.equal(a, b)
    with pytest.raises(N.SIError):
        N.call("si_qgemm", ctx.handle, w.handle, N.ptr(x), N.ptr(a), 0)
    w.free()


def test_cached_f16_weight_matches_the_oracle_too(ctx):
    """Q4_K without a cached copy is dequantised in shared memory (f16x2
    arithmetic); with si_qgemm_cache_weight the GEMM reads the f16 copy (f32
    arithmetic, one rounding).  Both stay within the bar of the oracle."""
    import torch
    blocks = synth_blocks_host(N.SI_Q4_K, 512, 1024, 8, 2, N.SYNTH_PLAIN, 0.01)
    xb, xf = bf16_round(np.random.default_rng(8).standard_normal((200, 1024)))
    ref = oracle.qmatvec(N.SI_Q4_K, blocks, 512, 1024, xf)
    w = ctx.upload(N.SI_Q4_K, blocks, 512, 1024)
    x = torch.from_numpy(xb.view(np.int16)).cuda().view(torch.bfloat16)
    a = ctx.qgemm(w, x).cpu().numpy()
    ctx.qgemm_cache_weight(w)
    b = ctx.qgemm(w, x).cpu().numpy()
    ctx.synchronize()
    assert rel_l2(a, ref) < TOL and rel_l2(b, ref) < TOL, (rel_l2(a, ref), rel_l2(b, ref))
    w.free()
