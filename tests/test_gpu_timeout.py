"""Failure detection without a GPU fault: a tensor-parallel rank that never
steps.  The device-side waits of the other rank are bounded (about a second,
the counterpart of WaitForResponseAsync's timeout, src/SharpInfer.Core/Engine/
DistributedInference.cs:158, :802); they give up, the step returns
SI_ERR_TIMEOUT, and the context keeps working.

Both ranks are models in this process on the one GPU, wired by their device
pointers (si_model_tp_connect_local).  Only rank 0 is ever stepped, so no two
kernels wait on each other: rank 0's waits run out on words nobody writes."""
import time

import numpy as np
import pytest

import oracle
from conftest import rel_l2
from sharpinfer_b200 import native as N
from sharpinfer_b200.backend import synth_blocks_host, synth_f32_host

pytestmark = pytest.mark.gpu
SI_ERR_TIMEOUT = 6


def test_rank_that_never_steps_times_out_and_context_survives(ctx):
    import torch
    from sharpinfer_b200.model import DecodeModel, config
    cfg = config(2, 512, 1024, 8, 4, 512, 96, 1)
    ranks = [DecodeModel(ctx, cfg, tp=2, rank=r) for r in range(2)]
    for m in ranks:
        m.synth(5)
        m.kv_synth(16, 5)
    for m in ranks:
        m.tp_connect_local(ranks)
    for attempt in range(2):  # the first step also captures the graph
        t0 = time.time()
        with pytest.raises(N.SIError) as ei:
            ranks[0].step([3], 16 + attempt)
        dt = time.time() - t0
        assert ei.value.status == SI_ERR_TIMEOUT, str(ei.value)
        assert dt < 10.0, dt  # one ~1 s timeout per step, not one per awaited word
    # the context still computes correctly, and its error word was cleared
    blocks = synth_blocks_host(N.SI_Q4_K, 256, 512, 9, 1, N.SYNTH_PLAIN, 0.01)
    x = synth_f32_host(512, 9, 2).reshape(1, 512)
    w = ctx.upload(N.SI_Q4_K, blocks, 256, 512)
    for _ in range(2):
        y = ctx.qmatvec(w, torch.from_numpy(x).cuda()).cpu().numpy()
        ctx.synchronize()
        assert rel_l2(y, oracle.qmatvec(N.SI_Q4_K, blocks, 256, 512, x)) < 1e-3
    w.free()
    for m in ranks:
        m.free()


def test_connect_local_rejects_mismatched_ranks(ctx):
    from sharpinfer_b200.model import DecodeModel, config
    a = DecodeModel(ctx, config(1, 512, 1024, 8, 4, 512, 64, 1), tp=2, rank=0)
    b = DecodeModel(ctx, config(1, 512, 1024, 8, 4, 512, 64, 1), tp=2, rank=0)
    with pytest.raises(N.SIError):
        a.tp_connect_local([a, b])  # entry 1 is not rank 1
    a.free()
    b.free()
