"""si_qmatvec_noalloc (the matvec with a fixed in-library scratch array) against
the allocating entry point si_qmatvec, through the C ABI.

Collected last (file name) so that it also runs after every other GPU test in
the same process; it must pass alone in a fresh process as well.
"""
import numpy as np
import pytest

from conftest import rel_l2
from sharpinfer_b200 import native as N

pytestmark = pytest.mark.gpu
TOL = 2e-5  # the matvec parity tolerance of test_gpu_quant.py
SI_ERR_UNSUPPORTED = 4  # si_status, include/sharpinfer_b200.h

CASES = [
    (N.SI_Q4_K, 4096, 4096, 1),    # streaming kernel, split row tiles
    (N.SI_Q6_K, 1000, 768, 3),     # ragged rows
    (N.SI_Q8_0, 2384, 512, 5),     # batch > 4: global-memory kernel
    (N.SI_Q4_K, 14336, 4096, 16),  # largest batch
    (N.SI_Q4_K, 32768, 16384, 4),  # the stated maximum shape
]


def noalloc(w, x, y, batch, stream):
    N.call("si_qmatvec_noalloc", w.handle, N.ptr(x), N.ptr(y), batch, stream)


@pytest.mark.parametrize("qt,rows,cols,batch", CASES)
def test_noalloc_matches_qmatvec(ctx, qt, rows, cols, batch):
    import torch
    w = ctx.synth_weight(qt, rows, cols, 11, 3, N.SYNTH_PLAIN, 0.01)
    g = torch.Generator(device="cpu").manual_seed(rows + cols + batch)
    x = torch.randn(batch, cols, generator=g).cuda()
    ref = ctx.qmatvec(w, x)
    torch.cuda.synchronize()
    ref = ref.cpu().numpy()
    side = torch.cuda.Stream()
    for call in range(2):  # two calls in a row share the scratch array
        y = torch.full((batch, rows), float("nan"), device="cuda")
        torch.cuda.synchronize()
        noalloc(w, x, y, batch, side.cuda_stream)
        out = y.cpu().numpy()
        assert np.isfinite(out).all(), call
        assert rel_l2(out, ref) <= TOL, (call, rel_l2(out, ref))
    w.free()


def test_noalloc_default_stream(ctx):
    import torch
    w = ctx.synth_weight(N.SI_Q4_K, 512, 1024, 5, 9, N.SYNTH_PLAIN, 0.01)
    x = torch.randn(2, 1024).cuda()
    ref = ctx.qmatvec(w, x)
    torch.cuda.synchronize()
    y = torch.empty(2, 512, device="cuda")
    noalloc(w, x, y, 2, None)
    assert rel_l2(y.cpu().numpy(), ref.cpu().numpy()) <= TOL
    w.free()


@pytest.mark.parametrize("rows,cols", [(32784, 256), (16, 16640)])
def test_noalloc_rejects_shapes_above_the_limit(ctx, rows, cols):
    import torch
    w = ctx.synth_weight(N.SI_Q4_K, rows, cols, 1, 1, N.SYNTH_PLAIN, 0.01)
    x = torch.zeros(1, cols, device="cuda")
    y = torch.zeros(1, rows, device="cuda")
    with pytest.raises(N.SIError) as e:
        noalloc(w, x, y, 1, None)
    assert e.value.status == SI_ERR_UNSUPPORTED and "limit" in str(e.value)
    with pytest.raises(N.SIError):
        noalloc(w, x, y, 17, None)
    w.free()
