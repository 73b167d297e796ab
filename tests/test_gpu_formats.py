"""Q4_0, Q2_K, Q3_K and Q5_K on the GPU: dequantisation bit for bit against
gguf-py's decoders (tests/golden/dequant_more.npz), the matvec at batch 1, 4
and 16 and the prefill GEMM against the oracle's dequantise-then-Dot
(TensorOps.MatVecMul / MatMul, src/SharpInfer.Core/Tensors/TensorOps.cs:63-112),
and the no-allocation entry point on these formats.  Bars: bit-exact for
dequantisation, relative L2 1e-5 for the f32 matvec, 1e-3 for the f16 GEMM."""
import os

import numpy as np
import pytest

import oracle
from conftest import GOLDEN, rel_l2
from sharpinfer_b200 import native as N

pytestmark = pytest.mark.gpu
G = np.load(os.path.join(GOLDEN, "dequant_more.npz"))
BB = {2: (32, 18), 10: (256, 84), 11: (256, 110), 13: (256, 176)}
QTS = [N.SI_Q4_0, N.SI_Q2_K, N.SI_Q3_K, N.SI_Q5_K]


def canon(a):
    bits = np.asarray(a, np.float32).view(np.uint32).copy()
    bits[np.isnan(a)] = 0x7FC00000
    return bits


def random_blocks(qt, rows, cols, seed):
    """GGUF blocks with finite scales (the golden generator's recipe)."""
    be, bb = BB[qt]
    rng = np.random.default_rng(seed)
    nb = rows * cols // be
    b = rng.integers(0, 256, (nb, bb)).astype(np.uint8)
    offs = {2: (0,), 10: (80, 82), 11: (108,), 13: (0, 2)}[qt]
    for off in offs:
        d = (np.abs(rng.standard_normal(nb)) * 0.01).astype(np.float16).view(np.uint8).reshape(nb, 2)
        b[:, off:off + 2] = d
    return b.ravel()


@pytest.mark.parametrize("qt", QTS)
@pytest.mark.parametrize("case", ["plain", "edge"])
def test_dequant_bit_exact_vs_gguf_py(ctx, qt, case):
    blk = G["t%d_%s_blocks" % (qt, case)]
    want = G["t%d_%s_bits" % (qt, case)]
    n = want.size
    w = ctx.upload(qt, blk, n // 256, 256)
    got = ctx.dequant(w).cpu().numpy().ravel()
    ctx.synchronize()
    with np.errstate(invalid="ignore"):
        assert np.array_equal(canon(got), want)
    w.free()


@pytest.mark.parametrize("qt", QTS)
@pytest.mark.parametrize("B", [1, 4, 16])
def test_matvec_matches_oracle(ctx, qt, B):
    import torch
    rows, cols = 300, 1024
    blk = random_blocks(qt, rows, cols, qt * 10 + B)
    x = np.random.default_rng(B).standard_normal((B, cols)).astype(np.float32)
    w = ctx.upload(qt, blk, rows, cols)
    y = ctx.qmatvec(w, torch.from_numpy(x).cuda()).cpu().numpy()
    ctx.synchronize()
    ref = oracle.qmatvec(qt, blk, rows, cols, x)
    assert rel_l2(y, ref) < 1e-5, rel_l2(y, ref)
    # the host-buffer and no-allocation entry points give the same values
    yh = ctx.qmatvec_host(w, x)
    assert rel_l2(yh, ref) < 1e-5
    y2 = torch.empty((B, rows), device="cuda")
    N.call("si_qmatvec_noalloc", w.handle, N.ptr(torch.from_numpy(x).cuda()), N.ptr(y2), B, None)
    assert np.array_equal(y2.cpu().numpy(), y)
    w.free()


@pytest.mark.parametrize("qt", QTS)
def test_prefill_gemm_matches_oracle(ctx, qt):
    import torch
    rows, cols, M = 384, 512, 200
    blk = random_blocks(qt, rows, cols, qt)
    b = np.random.default_rng(qt).standard_normal((M, cols)).astype(np.float32).view(np.uint32)
    xb = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    xf = (xb.astype(np.uint32) << 16).view(np.float32)
    w = ctx.upload(qt, blk, rows, cols)
    y = ctx.qgemm(w, torch.from_numpy(xb.view(np.int16)).cuda().view(torch.bfloat16)).cpu().numpy()
    ctx.synchronize()
    ref = oracle.qmatvec(qt, blk, rows, cols, xf)
    assert rel_l2(y, ref) < 1e-3, rel_l2(y, ref)
    w.free()
