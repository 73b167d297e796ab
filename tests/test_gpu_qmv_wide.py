"""Batch 5..16 Q4_K / Q6_K matvec over 256-row blocks (k_qmv_wide) against
the oracle's TensorOps.MatVecMul (src/SharpInfer.Core/Tensors/TensorOps.cs:20-72)
over the dequantised weights (Quantization.cs:273-314, 362-398).

Shapes cover: row counts that are not a multiple of the 256-row block (the
last block partly empty, odd tile counts), row blocks whose units are split
between CTAs (combined by the last CTA to arrive), the Llama-3-8B gate/up,
down and lm_head shapes and a 70B tensor-parallel vocabulary slice (16032
rows)."""
import numpy as np
import pytest

import oracle
from conftest import rel_l2
from sharpinfer_b200 import native as N
from sharpinfer_b200.backend import synth_blocks_host, synth_f32_host

pytestmark = pytest.mark.gpu
Q4K = N.SI_Q4_K


@pytest.fixture(autouse=True)
def _force_wide(monkeypatch):
    """Route every shape to k_qmv_wide (by default it takes 7168 rows and up)."""
    monkeypatch.setenv("SHARPINFER_B200_QMV_WIDE", "2")
QTS = [N.SI_Q4_K, N.SI_Q6_K]


def _run(ctx, rows, cols, batch, seed=77, scale=1.0, qt=Q4K):
    import torch
    blocks = synth_blocks_host(qt, rows, cols, seed, 3, N.SYNTH_PLAIN, 0.01)
    x = (synth_f32_host(batch * cols, seed, 100 + batch).reshape(batch, cols) * np.float32(scale)).astype(np.float32)
    ref = oracle.qmatvec(qt, blocks, rows, cols, x)
    w = ctx.upload(qt, blocks, rows, cols)
    y = ctx.qmatvec(w, torch.from_numpy(x).cuda())
    ctx.synchronize()
    return y.cpu().numpy(), ref, w, x


@pytest.mark.parametrize("qt", QTS)
@pytest.mark.parametrize("batch", [5, 7, 8, 9, 12, 13, 16])
@pytest.mark.parametrize("rows,cols", [(16, 256), (200, 512), (1040, 1024), (4096, 4096), (16032, 1024)])
def test_wide_matvec_parity(ctx, rows, cols, batch, qt):
    y, ref, _, _ = _run(ctx, rows, cols, batch, qt=qt)
    for b in range(batch):
        assert rel_l2(y[b], ref[b]) < 2e-5, (b, rel_l2(y[b], ref[b]))


@pytest.mark.parametrize("rows,cols,qt", [(28672, 4096, Q4K), (4096, 14336, Q4K), (128256, 4096, N.SI_Q6_K)])
def test_wide_matvec_llama8b_shapes_batch16(ctx, rows, cols, qt):
    y, ref, _, _ = _run(ctx, rows, cols, 16, seed=5, qt=qt)
    assert rel_l2(y, ref) < 2e-5


@pytest.mark.parametrize("qt", QTS)
def test_wide_matvec_is_deterministic(ctx, qt):
    import torch
    rows, cols, batch = 4096, 4096, 16
    w = ctx.synth_weight(qt, rows, cols, 3, 4)
    x = torch.from_numpy(synth_f32_host(batch * cols, 3, 5).reshape(batch, cols)).cuda()
    ys = [ctx.qmatvec(w, x).cpu().numpy() for _ in range(3)]
    ctx.synchronize()
    assert np.array_equal(ys[0], ys[1]) and np.array_equal(ys[1], ys[2])


@pytest.mark.parametrize("scale", [1e-20, 3e3, 1e30])
def test_wide_matvec_activation_range(ctx, scale):
    y, ref, _, _ = _run(ctx, 512, 1024, 11, seed=9, scale=scale)
    assert rel_l2(y, ref) < 2e-5


def test_wide_matvec_accumulates(ctx):
    """The residual-add epilogue: out += W x for every batch row."""
    import torch
    rows, cols, batch = 640, 2048, 13
    blocks = synth_blocks_host(Q4K, rows, cols, 1, 2, N.SYNTH_PLAIN, 0.01)
    x = synth_f32_host(batch * cols, 3, 4).reshape(batch, cols)
    w = ctx.upload(Q4K, blocks, rows, cols)
    ref = oracle.qmatvec(Q4K, blocks, rows, cols, x)
    base = torch.full((batch, rows), 2.0, device="cuda")
    ctx.synchronize()
    ctx.act_prepare(torch.from_numpy(x).cuda())
    ctx.qmatvec_prepared(w, batch, out=base, accumulate=True)
    ctx.synchronize()
    assert rel_l2(base.cpu().numpy(), ref + 2.0) < 2e-5
