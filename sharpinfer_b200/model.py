"""Decode model over the C ABI (si_model_*): a Llama/Mistral-architecture
transformer resident on one B200, stepped one token per sequence at a time
(Transformer.Forward, src/SharpInfer.Core/Layers/Transformer.cs:67-162).
"""
import ctypes

import numpy as np

from . import native as N


def config(n_layers, hidden, intermediate, n_heads, n_kv_heads, vocab, max_seq, max_batch=1,
           head_dim=128, rms_eps=1e-5, rope_theta=500000.0, weight_qtype=N.SI_Q4_K,
           lm_head_qtype=N.SI_Q6_K, emb_qtype=N.SI_Q4_K):
    return N.ModelConfig(n_layers, hidden, intermediate, n_heads, n_kv_heads, head_dim, vocab, max_seq,
                         max_batch, rms_eps, rope_theta, weight_qtype, lm_head_qtype, emb_qtype)


def llama3_8b(max_seq=4160, max_batch=1):
    """Llama-3-8B architecture: 32 layers, hidden 4096, 32 q / 8 kv heads, FFN 14336, vocab 128256."""
    return config(32, 4096, 14336, 32, 8, 128256, max_seq, max_batch)


def llama3_70b(max_seq=8256, max_batch=1):
    """Llama-3-70B architecture: 80 layers, hidden 8192, 64 q / 8 kv heads, FFN 28672, vocab 128256."""
    return config(80, 8192, 28672, 64, 8, 128256, max_seq, max_batch)


def tensor_recipe(cfg, layer, tensor):
    """(tag, qtype, recipe, sigma, mean, rows, cols) of a synthetic tensor."""
    tag, qt, rc = ctypes.c_uint64(), ctypes.c_int(), ctypes.c_int()
    sg, mu = ctypes.c_float(), ctypes.c_float()
    rows, cols = ctypes.c_int64(), ctypes.c_int64()
    N.call("si_model_tensor_recipe", ctypes.byref(cfg), layer, tensor, ctypes.byref(tag), ctypes.byref(qt),
           ctypes.byref(rc), ctypes.byref(sg), ctypes.byref(mu), ctypes.byref(rows), ctypes.byref(cols))
    return tag.value, qt.value, rc.value, sg.value, mu.value, rows.value, cols.value


def host_tensor(cfg, seed, layer, tensor):
    """Host bytes (GGUF blocks, or f32 norms) identical to what si_model_synth puts on the device."""
    from .backend import synth_blocks_host, synth_f32_host
    tag, qt, rc, sg, mu, rows, cols = tensor_recipe(cfg, layer, tensor)
    if qt == N.SI_F32:
        return synth_f32_host(cols, seed, tag, mu, sg)
    return synth_blocks_host(qt, rows, cols, seed, tag, rc, sg)


def host_kv(cfg, seed, layer, seq, length):
    """f16 K and V of cache positions [0, length) in the reference layout [pos][kv head][dim]."""
    from .backend import synth_f16_host
    n = length * cfg.n_kv_heads * cfg.head_dim
    lib = N.load()
    k = synth_f16_host(n, seed, lib.si_model_kv_tag(layer, seq, 0))
    v = synth_f16_host(n, seed, lib.si_model_kv_tag(layer, seq, 1))
    return k, v


def tp_slice(cfg, tp, rank, tensor):
    """(grow0, rows, gb0, nblk, gnblk): the part of a whole tensor rank `rank` of `tp` holds."""
    out = [ctypes.c_int64() for _ in range(5)]
    N.call("si_tp_slice", ctypes.byref(cfg), tp, rank, tensor, *[ctypes.byref(o) for o in out])
    return tuple(o.value for o in out)


def exchange_handles(handle, group=None):
    """Every rank's 64-byte buffer handle, in rank order, over torch.distributed."""
    import torch.distributed as dist
    got = [None] * dist.get_world_size(group)
    dist.all_gather_object(got, bytes(handle), group=group)
    return b"".join(got)


class DecodeModel:
    """si_model*: weights, f16 KV cache and the graph-captured decode step.
    With tp > 1 this is rank `rank` of a tensor-parallel model; connect it to
    the other ranks with tp_connect(exchange_handles(model.tp_handle()))."""

    def __init__(self, ctx, cfg, tp=1, rank=0):
        self.ctx, self.cfg, self.tp, self.rank = ctx, cfg, tp, rank
        h = ctypes.c_void_p()
        N.call("si_model_create_tp", ctx.handle, ctypes.byref(cfg), tp, rank, ctypes.byref(h))
        self.handle = h
        ctx._adopt(self)

    @property
    def local_vocab(self):
        return self.cfg.vocab // self.tp

    def tp_handle(self):
        buf = ctypes.create_string_buffer(64)
        N.call("si_model_tp_handle", self.handle, buf, 64)
        return buf.raw

    def tp_connect(self, handles):
        N.call("si_model_tp_connect", self.handle, handles, len(handles))

    def tp_connect_local(self, ranks):
        """Connect to the other ranks' models living in this process (rank order)."""
        arr = (ctypes.c_void_p * len(ranks))(*[r.handle.value for r in ranks])
        N.call("si_model_tp_connect_local", self.handle, arr, len(ranks))

    def free(self):
        if self.handle:
            N.call("si_model_free", self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass

    def synth(self, seed):
        N.call("si_model_synth", self.handle, seed)

    def set_tensor(self, layer, tensor, data):
        data = np.ascontiguousarray(data)
        N.call("si_model_set_tensor", self.handle, layer, tensor, N.ptr(data))

    def kv_synth(self, length, seed):
        N.call("si_model_kv_synth", self.handle, length, seed)

    def kv_write(self, layer, seq, pos0, k, v):
        k = np.ascontiguousarray(k, np.uint16)
        v = np.ascontiguousarray(v, np.uint16)
        n = k.size // (self.cfg.n_kv_heads * self.cfg.head_dim)
        N.call("si_model_kv_write", self.handle, layer, seq, pos0, n, N.ptr(k), N.ptr(v))

    def step(self, tokens, pos, logits=False):
        """Greedy next token of each sequence (and optionally the logits)."""
        tok = np.ascontiguousarray(tokens, np.int32).ravel()
        out = np.empty(tok.size, np.int32)
        lg = np.empty((tok.size, self.local_vocab), np.float32) if logits else None
        N.call("si_decode_step", self.handle, N.ptr(tok), tok.size, pos, N.ptr(out), N.ptr(lg))
        return (out, lg) if logits else out

    def generate(self, tokens, pos0, nsteps):
        """nsteps greedy tokens per sequence, decoded on the device: [nsteps][batch]."""
        tok = np.ascontiguousarray(tokens, np.int32).ravel()
        out = np.empty((nsteps, tok.size), np.int32)
        N.call("si_decode_generate", self.handle, N.ptr(tok), tok.size, pos0, nsteps, N.ptr(out))
        return out

    def prefill(self, tokens, pos0=0, seq=0, logits=False):
        """The prompt tokens of sequence `seq` at positions pos0.. through every
        layer at once (tensor-core GEMMs and causal flash attention), filling the
        KV cache; returns the greedy next token (and its logits)."""
        tok = np.ascontiguousarray(tokens, np.int32).ravel()
        out = np.empty(1, np.int32)
        lg = np.empty(self.local_vocab, np.float32) if logits else None
        N.call("si_model_prefill", self.handle, seq, N.ptr(tok), tok.size, pos0, N.ptr(out), N.ptr(lg))
        return (int(out[0]), lg) if logits else int(out[0])

    def kv_read(self, layer, seq, pos0, n):
        """f16 K and V of positions pos0 .. pos0 + n - 1 as [n][kv head][dim] (uint16)."""
        shape = (n, self.cfg.n_kv_heads // self.tp, self.cfg.head_dim)
        k = np.empty(shape, np.uint16)
        v = np.empty(shape, np.uint16)
        N.call("si_model_kv_read", self.handle, layer, seq, pos0, n, N.ptr(k), N.ptr(v))
        return k, v

    def kv_export(self, seq, length):
        """The prompt-cache byte format of KVCache.WriteRawData: per layer K then V, f32."""
        n = self.cfg.n_layers * 2 * length * self.cfg.n_kv_heads * self.cfg.head_dim
        out = np.empty(n, np.float32)
        N.call("si_model_kv_export", self.handle, seq, length, N.ptr(out), out.nbytes)
        return out

    def kv_import(self, seq, length, data):
        data = np.ascontiguousarray(data, np.float32)
        N.call("si_model_kv_import", self.handle, seq, length, N.ptr(data), data.nbytes)

    def step_kernels(self, batch=1):
        """Kernel launches in one captured decode step at this batch size."""
        n = ctypes.c_int()
        N.call("si_decode_step_kernels", self.handle, batch, ctypes.byref(n))
        return n.value

    def attention(self, layer, qkv, pos, out=None):
        """Attention of one layer for qkv [batch][(nh + 2 nkv) * hd] (CUDA f32 tensor)."""
        import torch
        batch = qkv.shape[0]
        if out is None:
            out = torch.empty((batch, self.cfg.n_heads * self.cfg.head_dim), dtype=torch.float32,
                              device=qkv.device)
        torch.cuda.synchronize()
        N.call("si_model_attention", self.handle, layer, N.ptr(qkv), N.ptr(out), batch, pos)
        return out
