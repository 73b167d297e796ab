"""Tensor-parallel decode on 2 GPUs (one process per GPU, peer-memory partial
sums) against the oracle's single-device forward pass
(Transformer.Forward, src/SharpInfer.Core/Layers/Transformer.cs:67-162):
identical greedy tokens, logits within 1e-3 relative L2 (the partial sums of
Wo / Wdown are added in rank order, a different summation order)."""
import os
import socket
import tempfile

import numpy as np
import pytest
import torch.multiprocessing as mp

import oracle
from conftest import rel_l2

pytestmark = pytest.mark.gpu
SEED = 11
CFG = (2, 1024, 1536, 8, 4, 1000, 320, 2)  # layers, hidden, FFN, heads, kv heads, vocab, max_seq, max_batch


def _gpus():
    import torch
    return torch.cuda.device_count()


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, kv_len, steps, starts, outdir):
    import torch
    import torch.distributed as dist
    from sharpinfer_b200 import B200Context
    from sharpinfer_b200.model import DecodeModel, config, exchange_handles
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.cuda.set_device(rank)
    ctx = B200Context(rank)
    m = DecodeModel(ctx, config(*CFG), tp=world, rank=rank)
    m.synth(SEED)
    m.tp_connect(exchange_handles(m.tp_handle()))
    res = {}
    for name, start in starts.items():
        m.kv_synth(kv_len, SEED)
        toks, T, L = list(start), [], []
        for s in range(steps):
            out, lg = m.step(toks, kv_len + s, logits=True)
            T.append(out.copy())
            L.append(lg.copy())
            toks = list(out)
        m.kv_synth(kv_len, SEED)
        res[name + "_tokens"] = np.array(T)
        res[name + "_logits"] = np.array(L)
        res[name + "_gen"] = m.generate(list(start), kv_len, steps)
    np.savez(os.path.join(outdir, "rank%d.npz" % rank), **res)
    dist.barrier()
    m.free()
    ctx.close()
    dist.destroy_process_group()


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
def test_tp2_decode_matches_oracle():
    from sharpinfer_b200.model import config
    kv_len, steps = 40, 4
    starts = {"b2": [5, 777], "b1": [42]}
    outdir = tempfile.mkdtemp()
    ctx = mp.get_context("spawn")
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, kv_len, steps, starts, outdir)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
    for p in procs:
        if p.is_alive():
            p.kill()
        assert p.exitcode == 0
    r0 = np.load(os.path.join(outdir, "rank0.npz"))
    r1 = np.load(os.path.join(outdir, "rank1.npz"))
    cfg = config(*CFG)
    for name, start in starts.items():
        assert np.array_equal(r0[name + "_tokens"], r1[name + "_tokens"])
        assert np.array_equal(r0[name + "_gen"], r0[name + "_tokens"])
        logits = np.concatenate([r0[name + "_logits"], r1[name + "_logits"]], axis=-1)  # vocabulary slices
        om = oracle.synthetic_model(cfg, SEED, n_seq=len(start), kv_len=kv_len)
        toks = list(start)
        for s in range(steps):
            for b in range(len(start)):
                ref = om.forward(b, toks[b], kv_len + s)
                assert rel_l2(logits[s, b], ref) < 1e-3, (name, s, b, rel_l2(logits[s, b], ref))
                assert r0[name + "_tokens"][s, b] == oracle.argmax(ref), (name, s, b)
            toks = list(r0[name + "_tokens"][s])
