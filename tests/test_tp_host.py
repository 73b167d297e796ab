"""Host side of tensor parallelism, no GPU: the shard plan (si_tp_slice) splits
every tensor exactly once across the ranks, and the buffer-handle exchange
works between processes (world size 2 over gloo on 127.0.0.1)."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from sharpinfer_b200 import native as N
from sharpinfer_b200.model import config, exchange_handles, llama3_70b, llama3_8b, tp_slice

TENSORS = [N.T_Q, N.T_K, N.T_V, N.T_O, N.T_GATE, N.T_UP, N.T_DOWN, N.T_EMB, N.T_LM_HEAD]


def whole(cfg, t):
    """(rows, blocks per row) of the whole tensor."""
    be = 32 if cfg.weight_qtype == N.SI_Q8_0 else 256
    h, hd = cfg.hidden, cfg.head_dim
    return {N.T_Q: (cfg.n_heads * hd, h // be), N.T_K: (cfg.n_kv_heads * hd, h // be),
            N.T_V: (cfg.n_kv_heads * hd, h // be), N.T_O: (h, cfg.n_heads * hd // be),
            N.T_GATE: (cfg.intermediate, h // be), N.T_UP: (cfg.intermediate, h // be),
            N.T_DOWN: (h, cfg.intermediate // be), N.T_EMB: (cfg.vocab, h // 256),
            N.T_LM_HEAD: (cfg.vocab, h // 256)}[t]


@pytest.mark.parametrize("name,cfg,tp", [("8b", llama3_8b(), 2), ("8b", llama3_8b(), 4), ("8b", llama3_8b(), 8),
                                         ("70b", llama3_70b(), 8),
                                         ("small", config(2, 1024, 1536, 8, 4, 1000, 320, 2), 2)])
def test_shards_cover_each_tensor_once(name, cfg, tp):
    for t in TENSORS:
        rows, nb = whole(cfg, t)
        cover = np.zeros((rows, nb), np.int32)
        for r in range(tp):
            g0, nr, b0, nbl, gnb = tp_slice(cfg, tp, r, t)
            assert gnb == nb
            cover[g0:g0 + nr, b0:b0 + nbl] += 1
        want = tp if t == N.T_EMB else 1  # the embedding is replicated
        assert (cover == want).all(), (name, t)


def test_slice_rejects_bad_rank():
    with pytest.raises(N.SIError):
        tp_slice(llama3_8b(), 2, 2, N.T_Q)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _exchange_worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        blob = bytes([rank * 16 + i % 16 for i in range(64)])
        q.put((rank, exchange_handles(blob)))
    finally:
        dist.destroy_process_group()


def test_handle_exchange_world2_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_exchange_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = b"".join(bytes([r * 16 + i % 16 for i in range(64)]) for r in range(2))
    assert got[0] == want and got[1] == want
