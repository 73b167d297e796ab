"""ctypes wrapper of the CPU oracle (oracle.cpp) -- TEST INFRASTRUCTURE ONLY.

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg,
and only as the checker or the timed CPU baseline; the sharpinfer_b200 package
never imports it.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_build", "liboracle.so")

_c_p = ctypes.c_void_p
_i32, _i64, _f32, _u16 = ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_uint16
_SIGS = {
    "or_half_to_float": (_f32, [_u16]),
    "or_block_size": (_i32, [_i32]),
    "or_block_bytes": (_i32, [_i32]),
    "or_dequant_tensor": (_i32, [_i32, _c_p, _i64, _c_p]),
    "or_dequant_reference_as_written": (_i32, [_i32, _c_p, _i64, _c_p]),
    "or_dot": (_f32, [_c_p, _c_p, _i32]),
    "or_matvec_f32": (None, [_c_p, _c_p, _c_p, _i64, _i32, _i32]),
    "or_qmatvec": (_i32, [_i32, _c_p, _i64, _i32, _c_p, _c_p, _i32, _i32]),
    "or_matmul": (None, [_c_p, _c_p, _c_p, _i32, _i32, _i32]),
    "or_softmax": (None, [_c_p, _i32]),
    "or_rmsnorm": (None, [_c_p, _c_p, _c_p, _i32, _f32]),
    "or_add_inplace": (None, [_c_p, _c_p, _i32]),
    "or_mul_inplace": (None, [_c_p, _c_p, _i32]),
    "or_silu": (None, [_c_p, _i32]),
    "or_add_scaled": (None, [_c_p, _c_p, _f32, _i32]),
    "or_argmax": (_i32, [_c_p, _i64]),
    "or_rope_apply": (None, [_c_p, _c_p, _i32, _i32, _i32, _i32, _f32]),
    "or_rope_table": (None, [_c_p, _i32, _i32, _f32]),
    "or_attention_decode": (None, [_c_p, _c_p, _c_p, _i32, _i32, _i32, _i32, _c_p, _i32]),
    "or_flash_attention": (None, [_c_p, _c_p, _c_p, _c_p, _i32, _i32, _i32, _f32, _i32, _i32]),
    "or_model_create": (_c_p, [_i32] * 8 + [_f32, _f32, _i32, _i32]),
    "or_model_free": (None, [_c_p]),
    "or_model_set": (None, [_c_p, _i32, _i32, _i32, _c_p]),
    "or_model_kv_fill": (None, [_c_p, _i32, _i32, _c_p, _c_p, _i32]),
    "or_model_forward": (_i32, [_c_p, _i32, _i32, _i32, _i32, _c_p]),
    "or_round_f16": (_f32, [_f32]),
    "or_model_kv_get": (None, [_c_p, _i32, _i32, _i32, _c_p, _c_p]),
    "or_num_threads": (_i32, []),
    "or_synth_blocks": (_i32, [_i32, _i64, _i64, ctypes.c_uint64, ctypes.c_uint64, _i32, _f32, _c_p]),
    "or_synth_f32": (None, [_i64, ctypes.c_uint64, ctypes.c_uint64, _f32, _f32, _c_p]),
    "or_synth_f16": (None, [_i64, ctypes.c_uint64, ctypes.c_uint64, _f32, _c_p]),
}

_lib = None


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def load():
    global _lib
    if _lib is None:
        srcs = [os.path.join(HERE, f) for f in ("oracle.cpp", "synth_host.cpp")]
        if not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(f) for f in srcs):
            build()
        lib = ctypes.CDLL(LIB)
        for n, (r, a) in _SIGS.items():
            f = getattr(lib, n)
            f.restype, f.argtypes = r, a
        _lib = lib
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data


def nthreads():
    return os.cpu_count() or 1


def dequant(qtype, blocks, n):
    out = np.empty(n, dtype=np.float32)
    rc = load().or_dequant_tensor(qtype, _p(np.ascontiguousarray(blocks, np.uint8)), n, _p(out))
    if rc:
        raise ValueError("oracle: unsupported type %d" % qtype)
    return out


def dequant_reference_as_written(qtype, blocks, nblocks):
    """The reference's own Q2_K / Q3_K / Q5_K decoders exactly as written
    (their field offsets differ from GGML's); 256 values per block."""
    out = np.empty(nblocks * 256, dtype=np.float32)
    if load().or_dequant_reference_as_written(qtype, _p(np.ascontiguousarray(blocks, np.uint8)), nblocks, _p(out)):
        raise ValueError("oracle: unsupported type %d" % qtype)
    return out


def dot(a, b):
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    return load().or_dot(_p(a), _p(b), a.size)


def qmatvec(qtype, blocks, rows, cols, x, threads=None):
    x = np.ascontiguousarray(x, np.float32).reshape(-1, cols)
    y = np.empty((x.shape[0], rows), np.float32)
    rc = load().or_qmatvec(qtype, _p(np.ascontiguousarray(blocks, np.uint8)), rows, cols, _p(x), _p(y),
                           x.shape[0], threads or nthreads())
    if rc:
        raise ValueError("oracle qmatvec failed")
    return y


def matvec_f32(W, x, threads=None):
    W = np.ascontiguousarray(W, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty(W.shape[0], np.float32)
    load().or_matvec_f32(_p(W), _p(x), _p(y), W.shape[0], W.shape[1], threads or nthreads())
    return y


def rmsnorm(x, w, eps):
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    load().or_rmsnorm(_p(out), _p(x), _p(np.ascontiguousarray(w, np.float32)), x.size, eps)
    return out


def softmax(x):
    x = np.array(x, np.float32)
    load().or_softmax(_p(x), x.size)
    return x


def silu(x):
    x = np.array(x, np.float32)
    load().or_silu(_p(x), x.size)
    return x


def argmax(x):
    x = np.ascontiguousarray(x, np.float32)
    return load().or_argmax(_p(x), x.size)


def rope_apply(q, k, pos, hd, theta):
    q = np.array(q, np.float32)
    k = np.array(k, np.float32)
    load().or_rope_apply(_p(q), _p(k), pos, hd, q.size // hd, k.size // hd, theta)
    return q, k


def rope_table(npos, hd, theta):
    t = np.empty(npos * hd, np.float32)
    load().or_rope_table(_p(t), npos, hd, theta)
    return t


def attention_decode(q, K, V, nh, nkv, hd, threads=None):
    q = np.ascontiguousarray(q, np.float32)
    K = np.ascontiguousarray(K, np.float32)
    V = np.ascontiguousarray(V, np.float32)
    kv_len = K.size // (nkv * hd)
    out = np.empty(nh * hd, np.float32)
    load().or_attention_decode(_p(q), _p(K), _p(V), kv_len, nh, nkv, hd, _p(out), threads or nthreads())
    return out


def flash_attention(Q, K, V, scale, causal, start_pos=0):
    Q = np.ascontiguousarray(Q, np.float32)
    K = np.ascontiguousarray(K, np.float32)
    V = np.ascontiguousarray(V, np.float32)
    seq, hd = Q.shape
    out = np.empty_like(Q)
    load().or_flash_attention(_p(Q), _p(K), _p(V), _p(out), seq, K.shape[0], hd, scale, int(causal), start_pos)
    return out


def matmul(a, b):
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    M, K = a.shape
    N = b.shape[1]
    c = np.empty((M, N), np.float32)
    load().or_matmul(_p(a), _p(b), _p(c), M, K, N)
    return c


def round_f16(x):
    return load().or_round_f16(x)


class OracleModel:
    """The reference forward pass (or_model_*, Transformer.Forward) over host GGUF tensors."""

    QKVO = ("q", "k", "v", "o", "gate", "up", "down")

    def __init__(self, cfg, n_seq, threads=None):
        L = load()
        self.cfg = cfg
        self.handle = L.or_model_create(cfg.n_layers, cfg.hidden, cfg.intermediate, cfg.n_heads, cfg.n_kv_heads,
                                        cfg.head_dim, cfg.vocab, cfg.max_seq, cfg.rms_eps, cfg.rope_theta, n_seq,
                                        threads or nthreads())
        if not self.handle:
            raise ValueError("oracle: hidden size must equal heads x head_dim (Transformer.cs:50)")
        self.keep = []

    def set(self, layer, which, qtype, data):
        data = np.ascontiguousarray(data)
        self.keep.append(data)
        load().or_model_set(self.handle, layer, which, qtype, _p(data))

    def kv_fill(self, seq, layer, k, v):
        k = np.ascontiguousarray(k, np.uint16)
        v = np.ascontiguousarray(v, np.uint16)
        load().or_model_kv_fill(self.handle, seq, layer, _p(k), _p(v), k.size // (self.cfg.n_kv_heads * self.cfg.head_dim))

    def forward(self, seq, token, pos, kv_round_f16=True):
        logits = np.empty(self.cfg.vocab, np.float32)
        rc = load().or_model_forward(self.handle, seq, token, pos, int(kv_round_f16), _p(logits))
        if rc:
            raise ValueError("oracle forward failed (%d)" % rc)
        return logits

    def kv_get(self, seq, layer, length):
        """Cached K, V of positions [0, length): f32 [length][kv heads][dim]."""
        shape = (length, self.cfg.n_kv_heads, self.cfg.head_dim)
        k = np.empty(shape, np.float32)
        v = np.empty(shape, np.float32)
        load().or_model_kv_get(self.handle, seq, layer, length, _p(k), _p(v))
        return k, v

    def __del__(self):
        try:
            if self.handle:
                load().or_model_free(self.handle)
        except Exception:
            pass


# ---- seeded synthetic model (the inputs both sides are given) ----------------
# Tensor ids and quant-type ids of the library's C ABI (si_tensor, si_qtype).
T_Q, T_K, T_V, T_O, T_GATE, T_UP, T_DOWN, T_ATTN_NORM, T_FFN_NORM = range(9)
T_EMB, T_LM_HEAD, T_FINAL_NORM = 100, 101, 102
F32, Q8_0, Q4_K, Q6_K = 0, 8, 12, 14
PLAIN, MODEL = 0, 1
BLOCK = {Q4_K: (256, 144), Q6_K: (256, 210), Q8_0: (32, 34)}


def synth_blocks(qt, rows, cols, seed, tag, recipe, sigma):
    """Seeded GGUF blocks (the bytes of the library's si_synth_blocks_host)."""
    be, bb = BLOCK[qt]
    out = np.empty(rows * (cols // be) * bb, np.uint8)
    if load().or_synth_blocks(qt, rows, cols, seed, tag, recipe, sigma, _p(out)):
        raise ValueError("oracle: bad synthetic shape")
    return out


def synth_f32(n, seed, tag, mean, sigma):
    out = np.empty(n, np.float32)
    load().or_synth_f32(n, seed, tag, mean, sigma, _p(out))
    return out


def synth_f16(n, seed, tag, sigma=1.0):
    out = np.empty(n, np.uint16)
    load().or_synth_f16(n, seed, tag, sigma, _p(out))
    return out


def _recipe_sigma(qt, recipe, cols):
    rc = np.sqrt(np.float32(cols))  # binary32 arithmetic, as the library computes it
    if qt == Q4_K:
        return np.float32(1.0) / (np.float32(23.3) * rc) if recipe == MODEL else np.float32(0.01)
    if qt == Q6_K:
        return np.float32(1.0) / (np.float32(348.0) * rc)
    return np.float32(1.0) / (np.float32(73.9) * rc)


def tensor_recipe(cfg, layer, t):
    """(tag, qtype, recipe, sigma, mean, rows, cols) of a tensor of the seeded
    synthetic model -- the same table as the library's si_model_tensor_recipe
    (a CPU test checks that the two agree)."""
    hd = cfg.head_dim
    qr, kr = cfg.n_heads * hd, cfg.n_kv_heads * hd
    q, rc, mu, sg = cfg.weight_qtype, MODEL, np.float32(0), np.float32(0)
    if layer < 0:
        tag = t - T_EMB + 1
        if t == T_EMB:
            q, r, k = cfg.emb_qtype, cfg.vocab, cfg.hidden
        elif t == T_LM_HEAD:
            q, r, k, rc = cfg.lm_head_qtype, cfg.vocab, cfg.hidden, PLAIN
        elif t == T_FINAL_NORM:
            q, r, k = F32, 1, cfg.hidden
        else:
            raise ValueError("unknown global tensor %d" % t)
    else:
        tag = 1000 * (layer + 1) + t
        r, k = {T_Q: (qr, cfg.hidden), T_K: (kr, cfg.hidden), T_V: (kr, cfg.hidden), T_O: (cfg.hidden, qr),
                T_GATE: (cfg.intermediate, cfg.hidden), T_UP: (cfg.intermediate, cfg.hidden),
                T_DOWN: (cfg.hidden, cfg.intermediate), T_ATTN_NORM: (1, cfg.hidden),
                T_FFN_NORM: (1, cfg.hidden)}[t]
        if t in (T_ATTN_NORM, T_FFN_NORM):
            q = F32
    if q == F32:
        mu, sg, rc = np.float32(1.0), np.float32(0.01), 0
    elif t == T_EMB:
        sg = np.float32(1.0) / np.float32(23.3) if q == Q4_K else _recipe_sigma(q, rc, 1)
    else:
        sg = _recipe_sigma(q, rc, k)
    return tag, q, rc, float(sg), float(mu), r, k


def host_tensor(cfg, seed, layer, t):
    tag, qt, rc, sg, mu, rows, cols = tensor_recipe(cfg, layer, t)
    if qt == F32:
        return synth_f32(cols, seed, tag, mu, sg)
    return synth_blocks(qt, rows, cols, seed, tag, rc, sg)


def kv_tag(layer, seq, is_value):
    return 0x4B560000 + (layer * 64 + seq) * 2 + int(bool(is_value))


def host_kv(cfg, seed, layer, seq, length):
    """f16 K and V of cache positions [0, length) in the reference layout [pos][kv head][dim]."""
    n = length * cfg.n_kv_heads * cfg.head_dim
    return synth_f16(n, seed, kv_tag(layer, seq, 0)), synth_f16(n, seed, kv_tag(layer, seq, 1))


def synthetic_model(cfg, seed, n_seq, kv_len, threads=None):
    """OracleModel holding exactly the tensors and KV prefix that the library's
    si_model_synth / si_model_kv_synth put on the device (same generator, run
    here on the host)."""
    om = OracleModel(cfg, n_seq, threads)
    ids = [T_Q, T_K, T_V, T_O, T_GATE, T_UP, T_DOWN]
    for l in range(cfg.n_layers):
        for which, t in enumerate(ids):
            om.set(l, which, cfg.weight_qtype, host_tensor(cfg, seed, l, t))
        om.set(l, 7, 0, host_tensor(cfg, seed, l, T_ATTN_NORM))
        om.set(l, 8, 0, host_tensor(cfg, seed, l, T_FFN_NORM))
    om.set(-1, 0, cfg.emb_qtype, host_tensor(cfg, seed, -1, T_EMB))
    om.set(-1, 1, cfg.lm_head_qtype, host_tensor(cfg, seed, -1, T_LM_HEAD))
    om.set(-1, 2, 0, host_tensor(cfg, seed, -1, T_FINAL_NORM))
    if kv_len:
        for b in range(n_seq):
            for l in range(cfg.n_layers):
                k, v = host_kv(cfg, seed, l, b, kv_len)
                om.kv_fill(b, l, k, v)
    return om
