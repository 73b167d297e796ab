"""The CPU oracle against known answers and golden vectors (no GPU).

Known answers are derived by hand from the reference decoders
(src/SharpInfer.Core/Tensors/Quantization.cs) and TensorOps
(src/SharpInfer.Core/Tensors/TensorOps.cs); the golden vectors in
tests/golden/dequant.npz come from gguf-py (see make_golden.py).
"""
import os

import numpy as np
import pytest

import oracle
from conftest import GOLDEN, rel_l2
from sharpinfer_b200 import native as N


def f16(x):
    return int(np.array([x], np.float16).view(np.uint16)[0])


def canon(a):
    a = np.asarray(a, np.float32)
    bits = a.view(np.uint32).copy()
    bits[np.isnan(a)] = 0x7FC00000
    return bits


# ---- HalfToFloat (Quantization.cs:394-398) -------------------------------------
@pytest.mark.parametrize("bits,val", [
    (0x3C00, 1.0), (0xBC00, -1.0), (0x0001, 2.0 ** -24), (0x03FF, 1023 * 2.0 ** -24),
    (0x0400, 2.0 ** -14), (0x7BFF, 65504.0), (0x7C00, np.inf), (0xFC00, -np.inf), (0x3555, 0.333251953125),
])
def test_half_to_float(bits, val):
    assert oracle.load().or_half_to_float(bits) == np.float32(val)


def test_half_to_float_signed_zero_and_nan():
    L = oracle.load()
    z = np.float32(L.or_half_to_float(0x8000))
    assert z == 0.0 and np.signbit(z)
    assert np.isnan(L.or_half_to_float(0x7E00))
    # every finite half converts exactly (compare with numpy's exact conversion)
    allh = np.arange(0, 65536, dtype=np.uint16)
    ref = allh.view(np.float16).astype(np.float32)
    got = np.array([L.or_half_to_float(int(h)) for h in allh[::7]], np.float32)
    assert np.array_equal(canon(got), canon(ref[::7]))


# ---- Known-answer blocks ----------------------------------------------------------
def test_q4k_known_answers():
    b = np.zeros(144, np.uint8)
    b[0:2] = [0x00, 0x3C]  # d = 1.0
    b[2:4] = [0x00, 0x38]  # dmin = 0.5
    # scales: sc0=2, m0=3 (j<4 branch); j=4: sc=(s8&0xF)|((s0>>6)<<4), m=(s8>>4)|((s4>>6)<<4)
    b[4:16] = [0x42, 0, 0, 0, 0xC3, 0, 0, 0, 0x95, 0, 0, 0]
    b[16] = 0x5A  # qs[0]: low nibble 10 -> out[0], high nibble 5 -> out[32]
    b[16 + 64] = 0x7C  # qs[64] belongs to pair j=4: low 12 -> out[128], high 7 -> out[160]
    out = oracle.dequant(N.SI_Q4_K, b, 256)
    assert out[0] == 2 * 10 - 3 * 0.5        # sc0=0x42&63=2, m0=0xC3&63=3
    # sc1 = s[1]&63 = 0, m1 = s[5]&63 = 0
    assert out[32] == 0.0
    # j=4: sc = (0x95 & 0xF) | ((0x42 >> 6) << 4) = 5 | 16 = 21
    #      m  = (0x95 >> 4) | ((0xC3 >> 6) << 4) = 9 | 48 = 57
    assert out[128] == 21 * 12 - 57 * 0.5
    # j=5: sc = (s9 & 0xF) | ((s1 >> 6) << 4) = 0, m = (s9 >> 4) | ((s5 >> 6) << 4) = 0
    assert out[160] == 0.0
    assert out[1] == 2 * 0 - 1.5


def test_q6k_known_answers():
    b = np.zeros(210, np.uint8)
    b[208:210] = [0x00, 0x40]  # d = 2.0
    sc = np.zeros(16, np.int8)
    sc[0], sc[2], sc[4], sc[6], sc[9] = 3, -128, 127, -1, 5
    b[192:208] = sc.view(np.uint8)
    b[0] = 0x2F      # ql[0]: low 15 -> q1 (l=0), high 2 -> q3
    b[32] = 0x91     # ql[32]: low 1 -> q2, high 9 -> q4
    b[128] = 0b11100100  # qh[0]: q1 hi=0, q2 hi=1, q3 hi=2, q4 hi=3
    b[64 + 17] = 0x0A   # second half, l=17: ql[64+17] low 10 -> out[128+17]
    b[128 + 32 + 17] = 0x03  # qh for second half l=17: hi=3 for q1
    out = oracle.dequant(N.SI_Q6_K, b, 256)
    assert out[0] == 2.0 * 3 * (15 - 32)
    assert out[32] == 2.0 * -128 * ((1 | 16) - 32)
    assert out[64] == 2.0 * 127 * ((2 | 32) - 32)
    assert out[96] == 2.0 * -1 * ((9 | 48) - 32)
    assert out[128 + 17] == 2.0 * 5 * ((10 | 48) - 32)  # scIdx = 8 + 17//16 = 9
    assert out[1] == 2.0 * 3 * (0 - 32)


def test_q80_known_answers():
    b = np.zeros(34, np.uint8)
    b[0:2] = [0x00, 0x34]  # d = 0.25
    b[2:] = np.arange(-16, 16, dtype=np.int8).view(np.uint8)
    b[2], b[3] = 0x80, 0x7F  # -128, 127
    out = oracle.dequant(N.SI_Q8_0, b, 32)
    assert out[0] == -32.0 and out[1] == 31.75
    assert np.array_equal(out[2:], (np.arange(-14, 16) * 0.25).astype(np.float32))


# ---- Golden vectors (gguf-py) -------------------------------------------------------
def golden_cases():
    z = np.load(os.path.join(GOLDEN, "dequant.npz"))
    names = sorted({k[:-5] for k in z.files if k.endswith("_meta")})
    return z, names


@pytest.mark.parametrize("name", golden_cases()[1])
def test_oracle_dequant_matches_golden(name):
    z, _ = golden_cases()
    qt, rows, cols = (int(v) for v in z[name + "_meta"])
    out = oracle.dequant(qt, z[name + "_blocks"], rows * cols).reshape(rows, cols)
    assert np.array_equal(canon(out), z[name + "_bits"]), name


def test_golden_generator_is_current():
    """The seeded blocks stored in the fixture are what the host generator makes today."""
    from sharpinfer_b200.backend import synth_blocks_host
    z, _ = golden_cases()
    assert np.array_equal(z["q4k_plain_blocks"], synth_blocks_host(N.SI_Q4_K, 24, 512, 1234, 1, N.SYNTH_PLAIN, 0.01))
    assert np.array_equal(z["q6k_plain_blocks"], synth_blocks_host(N.SI_Q6_K, 20, 512, 1234, 3, N.SYNTH_PLAIN, 0.01))
    assert np.array_equal(z["q80_plain_blocks"], synth_blocks_host(N.SI_Q8_0, 18, 256, 1234, 4, N.SYNTH_PLAIN, 0.01))


def test_oracle_dequant_random_vs_gguf():
    gguf = pytest.importorskip("gguf")
    from gguf import quants
    from sharpinfer_b200.backend import synth_blocks_host
    gt = {N.SI_Q4_K: gguf.GGMLQuantizationType.Q4_K, N.SI_Q6_K: gguf.GGMLQuantizationType.Q6_K,
          N.SI_Q8_0: gguf.GGMLQuantizationType.Q8_0}
    for qt in gt:
        for recipe in (N.SYNTH_PLAIN, N.SYNTH_MODEL):
            blocks = synth_blocks_host(qt, 64, 1024, 99, 5 + recipe, recipe, 0.05)
            ours = oracle.dequant(qt, blocks, 64 * 1024)
            ref = quants.dequantize(blocks.reshape(-1, N.BLOCK_BYTES[qt]), gt[qt]).astype(np.float32).ravel()
            assert np.array_equal(canon(ours), canon(ref))


# ---- TensorOps ----------------------------------------------------------------------
def test_dot_lane_order():
    """Dot (TensorOps.cs:20-57) sums 8 lanes, then (v4+v0, v5+v1, v6+v2, v7+v3) pairwise, then a scalar tail."""
    a = np.array([1e8, 1, 1, 1, -1e8, 1, 1, 1, 3, 0.5, 1, 1, 7, 1, 1, 1, 0.25, 0.125], np.float32)
    b = np.ones_like(a)
    v = np.zeros(8, np.float32)
    for i in range(0, 16, 8):
        v = (v + a[i:i + 8] * b[i:i + 8]).astype(np.float32)
    s = (v[4:] + v[:4]).astype(np.float32)
    h = np.float32(np.float32(s[0] + s[1]) + np.float32(s[2] + s[3]))
    for i in range(16, 18):
        h = np.float32(h + np.float32(a[i] * b[i]))
    assert oracle.dot(a, b) == h
    # the sequential sum differs: the lane order is observable
    seq = np.float32(0)
    for x in a:
        seq = np.float32(seq + x)
    assert seq != h


def test_qmatvec_equals_dequant_then_matvec():
    from sharpinfer_b200.backend import synth_blocks_host, synth_f32_host
    blocks = synth_blocks_host(N.SI_Q4_K, 33, 768, 3, 9, N.SYNTH_PLAIN, 0.01)
    W = oracle.dequant(N.SI_Q4_K, blocks, 33 * 768).reshape(33, 768)
    x = synth_f32_host(2 * 768, 3, 10)
    y = oracle.qmatvec(N.SI_Q4_K, blocks, 33, 768, x)
    for b in range(2):
        assert np.array_equal(y[b], oracle.matvec_f32(W, x[b * 768:(b + 1) * 768]))


def test_rmsnorm_softmax_silu_argmax():
    x = np.array([1.0, -2.0, 3.0, 0.5], np.float32)
    w = np.array([1.0, 0.5, 2.0, 1.0], np.float32)
    ss = np.float32(0)
    for v in x:
        ss = np.float32(ss + np.float32(v * v))
    scale = np.float32(1) / np.float32(np.sqrt(np.float32(ss / np.float32(4) + np.float32(1e-5))))
    assert np.array_equal(oracle.rmsnorm(x, w, 1e-5), (x * scale * w).astype(np.float32))
    p = oracle.softmax(x)
    assert abs(float(p.sum()) - 1.0) < 1e-6 and int(np.argmax(p)) == 2
    s = oracle.silu(np.array([0.0, 1.0], np.float32))
    assert s[0] == 0.0 and abs(s[1] - 1 / (1 + np.exp(-1.0))) < 1e-7
    # ArgMax: first index of the maximum (strict >), TensorOps.cs:221-234
    assert oracle.argmax(np.array([1, 5, 5, 2], np.float32)) == 1
    assert oracle.argmax(np.array([-np.inf, -np.inf], np.float32)) == 0


def test_flash_attention_matches_naive():
    rng = np.random.default_rng(0)
    for seq, kv, causal, start in [(70, 70, True, 0), (5, 130, True, 125), (64, 100, False, 0), (1, 1, True, 0)]:
        Q = rng.standard_normal((seq, 32)).astype(np.float32)
        K = rng.standard_normal((kv, 32)).astype(np.float32)
        V = rng.standard_normal((kv, 32)).astype(np.float32)
        out = oracle.flash_attention(Q, K, V, 1 / np.sqrt(32), causal, start)
        S = (Q.astype(np.float64) @ K.T.astype(np.float64)) / np.sqrt(32)
        if causal:
            qpos = start + np.arange(seq)[:, None]
            S = np.where(np.arange(kv)[None, :] > qpos, -np.inf, S)
        P = np.exp(S - S.max(1, keepdims=True))
        P /= P.sum(1, keepdims=True)
        assert rel_l2(out, P @ V) < 1e-5


def test_attention_decode_matches_naive():
    rng = np.random.default_rng(1)
    nh, nkv, hd, T = 8, 2, 64, 37
    q = rng.standard_normal(nh * hd).astype(np.float32)
    K = rng.standard_normal((T, nkv, hd)).astype(np.float32)
    V = rng.standard_normal((T, nkv, hd)).astype(np.float32)
    out = oracle.attention_decode(q, K, V, nh, nkv, hd).reshape(nh, hd)
    for h in range(nh):
        kvh = h // (nh // nkv)
        s = K[:, kvh, :].astype(np.float64) @ q[h * hd:(h + 1) * hd] / np.sqrt(hd)
        p = np.exp(s - s.max())
        p /= p.sum()
        assert rel_l2(out[h], p @ V[:, kvh, :]) < 1e-5


def test_rope_table_matches_apply():
    hd, theta = 128, 500000.0
    tab = oracle.rope_table(50, hd, theta).reshape(50, hd // 2, 2)
    rng = np.random.default_rng(2)
    q = rng.standard_normal(2 * hd).astype(np.float32)
    k = rng.standard_normal(hd).astype(np.float32)
    for pos in (0, 1, 49):
        q2, _ = oracle.rope_apply(q, k, pos, hd, theta)
        c, s = tab[pos, :, 0], tab[pos, :, 1]
        for h in range(2):
            x0, x1 = q[h * hd::2][:hd // 2], q[h * hd + 1::2][:hd // 2]
            e0 = (x0 * c - x1 * s).astype(np.float32)
            e1 = (x0 * s + x1 * c).astype(np.float32)
            assert np.array_equal(q2[h * hd:(h + 1) * hd:2], e0)
            assert np.array_equal(q2[h * hd + 1:(h + 1) * hd:2], e1)


def test_round_f16():
    for v in [1.0, 1.0 + 2 ** -11, 1.0 + 3 * 2 ** -11, 65519.0, 65520.0, 1e-8, 3e-5, -2.5]:
        assert oracle.round_f16(v) == np.float32(np.float16(v)) or (np.isinf(np.float16(v)) and np.isinf(oracle.round_f16(v)))
