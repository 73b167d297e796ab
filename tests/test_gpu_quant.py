"""GPU parity of the quantised weight path through the C ABI.

Dequantisation must be bit-exact with the oracle and the golden vectors
(Quantization.cs); the fused matvec must match the oracle's
TensorOps.MatVecMul over the dequantised weights within 1e-3 relative L2
(the tolerance the task states for matvec/GEMM outputs).
"""
import os

import numpy as np
import pytest

import oracle
from conftest import GOLDEN, rel_l2
from sharpinfer_b200 import native as N
from sharpinfer_b200.backend import synth_blocks_host, synth_f32_host

pytestmark = pytest.mark.gpu
TOL = 1e-3
QTS = [N.SI_Q4_K, N.SI_Q6_K, N.SI_Q8_0]


def canon(a):
    a = np.asarray(a, np.float32)
    bits = a.view(np.uint32).copy()
    bits[np.isnan(a)] = 0x7FC00000
    return bits


def golden_names():
    z = np.load(os.path.join(GOLDEN, "dequant.npz"))
    return sorted({k[:-5] for k in z.files if k.endswith("_meta")})


@pytest.mark.parametrize("name", golden_names())
def test_dequant_bit_exact_golden(ctx, name):
    z = np.load(os.path.join(GOLDEN, "dequant.npz"))
    qt, rows, cols = (int(v) for v in z[name + "_meta"])
    w = ctx.upload(qt, z[name + "_blocks"], rows, cols)
    out = ctx.dequant(w)
    ctx.synchronize()
    assert np.array_equal(canon(out.cpu().numpy()), z[name + "_bits"])


@pytest.mark.parametrize("qt", QTS)
@pytest.mark.parametrize("recipe", [N.SYNTH_PLAIN, N.SYNTH_MODEL])
def test_device_generator_matches_host(ctx, qt, recipe):
    rows, cols = 37, 512
    w = ctx.synth_weight(qt, rows, cols, 77, 3, recipe, 0.02)
    host = synth_blocks_host(qt, rows, cols, 77, 3, recipe, 0.02)
    got = ctx.dequant(w)
    ctx.synchronize()
    ref = oracle.dequant(qt, host, rows * cols).reshape(rows, cols)
    assert np.array_equal(canon(got.cpu().numpy()), canon(ref))


# Row tiles of 16; the streaming kernel splits the tiles' 256-column units
# evenly over one CTA per SM, so some shapes put a tile across two CTAs
# (e.g. 4800 x 768 and 4096 x 4096) and others do not (2384 x 256).
SHAPES = [(1, 256), (16, 256), (255, 512), (257, 1024), (2384, 256), (4800, 768), (4096, 4096),
          (1000, 14336)]


@pytest.mark.parametrize("qt", QTS)
@pytest.mark.parametrize("rows,cols", SHAPES)
@pytest.mark.parametrize("batch", [1, 3, 4, 5, 16])
def test_qmatvec_parity(ctx, qt, rows, cols, batch):
    import torch
    if batch == 16 and rows * cols > 4096 * 4096:
        pytest.skip("covered by smaller shapes")
    blocks = synth_blocks_host(qt, rows, cols, 1234, 10 + qt, N.SYNTH_PLAIN, 0.01)
    x = synth_f32_host(batch * cols, 1234, 500 + batch).reshape(batch, cols)
    ref = oracle.qmatvec(qt, blocks, rows, cols, x)
    w = ctx.upload(qt, blocks, rows, cols)
    y = ctx.qmatvec(w, torch.from_numpy(x).cuda())
    ctx.synchronize()
    err = rel_l2(y.cpu().numpy(), ref)
    assert err < TOL, err
    # much tighter than required: hi/lo activations keep f32-level accuracy
    assert err < 2e-5, err


@pytest.mark.parametrize("qt", QTS)
@pytest.mark.parametrize("batch", [1, 4, 7])
def test_qmatvec_is_deterministic(ctx, qt, batch):
    """Repeated calls give bit-identical results (shared row tiles are combined in a fixed order)."""
    import torch
    rows, cols = 4800, 768 if qt != N.SI_Q8_0 else 800
    w = ctx.synth_weight(qt, rows, cols, 3, 4)
    x = torch.from_numpy(synth_f32_host(batch * cols, 3, 5).reshape(batch, cols)).cuda()
    ys = [ctx.qmatvec(w, x).cpu().numpy() for _ in range(3)]
    ctx.synchronize()
    assert np.array_equal(ys[0], ys[1]) and np.array_equal(ys[1], ys[2])


@pytest.mark.parametrize("qt", QTS)
def test_qmatvec_host_entry_matches_device_entry(ctx, qt):
    import torch
    rows, cols, batch = 300, 1024, 2
    blocks = synth_blocks_host(qt, rows, cols, 5, 6, N.SYNTH_PLAIN, 0.01)
    x = synth_f32_host(batch * cols, 5, 7).reshape(batch, cols)
    w = ctx.upload(qt, blocks, rows, cols)
    yh = ctx.qmatvec_host(w, x)
    yd = ctx.qmatvec(w, torch.from_numpy(x).cuda())
    ctx.synchronize()
    assert np.array_equal(yh, yd.cpu().numpy())


@pytest.mark.parametrize("scale", [1e-20, 1e-3, 1.0, 3e3, 1e30])
def test_qmatvec_activation_dynamic_range(ctx, scale):
    """The per-vector power-of-two scaling keeps tiny and huge activations exact-ish."""
    import torch
    rows, cols = 64, 512
    blocks = synth_blocks_host(N.SI_Q4_K, rows, cols, 9, 9, N.SYNTH_PLAIN, 0.01)
    x = (synth_f32_host(cols, 9, 10) * np.float32(scale)).astype(np.float32)
    ref = oracle.qmatvec(N.SI_Q4_K, blocks, rows, cols, x)
    w = ctx.upload(N.SI_Q4_K, blocks, rows, cols)
    y = ctx.qmatvec(w, torch.from_numpy(x).cuda())
    ctx.synchronize()
    assert rel_l2(y.cpu().numpy(), ref) < 1e-5


def test_prepared_matvec_accumulates(ctx):
    import torch
    rows, cols = 128, 1024
    blocks = synth_blocks_host(N.SI_Q4_K, rows, cols, 1, 2, N.SYNTH_PLAIN, 0.01)
    x = synth_f32_host(cols, 3, 4)
    w = ctx.upload(N.SI_Q4_K, blocks, rows, cols)
    ref = oracle.qmatvec(N.SI_Q4_K, blocks, rows, cols, x)[0]
    base = torch.ones((1, rows), device="cuda")
    ctx.synchronize()
    ctx.act_prepare(torch.from_numpy(x).cuda().reshape(1, -1))
    ctx.qmatvec_prepared(w, 1, out=base, accumulate=True)
    ctx.synchronize()
    assert rel_l2(base.cpu().numpy()[0], ref + 1) < 1e-5


def test_invalid_arguments_raise(ctx):
    import torch
    w = ctx.synth_weight(N.SI_Q4_K, 16, 256, 1, 1)
    x = torch.zeros((17, 256), device="cuda")
    with pytest.raises(N.SIError) as e:
        ctx.qmatvec(w, x)
    assert e.value.status == 1
    with pytest.raises(N.SIError):
        ctx.synth_weight(N.SI_Q4_K, 16, 300, 1, 1)  # cols not a multiple of 256
    with pytest.raises(N.SIError):
        ctx.synth_weight(3, 16, 256, 1, 1)  # Q4_1 is not on this path
