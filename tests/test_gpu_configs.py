"""The hot-path kernels at the workload sizes the benchmark is quoted on, each
against the oracle:

* the prefill GEMM (si_qgemm) at M = 512 and 2048 tokens over the three
  Llama-3-8B projection shapes -- TensorOps.MatMul semantics
  (src/SharpInfer.Core/Tensors/TensorOps.cs:79-112) over the dequantised
  weights; a sample of 24 token rows is checked against the oracle's
  dequantise-then-Dot, and every row through a size-independent checksum
  (sum_r y[m][r] = x[m] . sum_r W[r], the right side in f64);
* bf16 activations over the whole range the type allows (|x| up to 1e5 and
  down to 1e-7 in one row, rows of zeros);
* prefill attention over 2048 causal tokens, 32 q / 8 kv heads
  (FlashAttention.Forward, src/SharpInfer.Core/Layers/FlashAttention.cs:59-167),
  a sample of heads;
* decode attention at 8192 cached positions with the Llama-3-70B head shape
  (64 q / 8 kv heads), Transformer.cs:94-129;
* greedy ArgMax ties: the first index of the maximum under strict '>'
  (SamplingPipeline.cs:83-89) through the whole decode step.
Bars: relative L2 1e-3 for the GEMM, 1e-4 for prefill attention, 1e-5 for
decode attention; token identity for ArgMax."""
import numpy as np
import pytest

import oracle
from conftest import rel_l2
from sharpinfer_b200 import native as N
from sharpinfer_b200.backend import synth_blocks_host
from sharpinfer_b200.model import DecodeModel, config, host_kv

pytestmark = pytest.mark.gpu


def bf16_round(a):
    b = np.ascontiguousarray(a, np.float32).view(np.uint32)
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    return r, (r.astype(np.uint32) << 16).view(np.float32)


def sample_rows(M):
    return np.unique(np.concatenate([np.arange(8), M // 2 - 4 + np.arange(8), M - 8 + np.arange(8)]))


@pytest.mark.parametrize("M", [512, 2048])
@pytest.mark.parametrize("rows,cols", [(4096, 4096), (14336, 4096), (4096, 14336)])
def test_prefill_gemm_llama8b_shapes(ctx, M, rows, cols):
    import torch
    blocks = synth_blocks_host(N.SI_Q4_K, rows, cols, 31, 7, N.SYNTH_MODEL, 1.0 / (23.3 * np.sqrt(cols)))
    rng = np.random.default_rng(M * 3 + rows)
    xb, xf = bf16_round(rng.standard_normal((M, cols)))
    w = ctx.upload(N.SI_Q4_K, blocks, rows, cols)
    x = torch.from_numpy(xb.view(np.int16)).cuda().view(torch.bfloat16)
    y = ctx.qgemm(w, x).cpu().numpy()
    ctx.synchronize()
    idx = sample_rows(M)
    ref = oracle.qmatvec(N.SI_Q4_K, blocks, rows, cols, xf[idx])
    err = rel_l2(y[idx], ref)
    assert err < 1e-3, err
    # checksum of every row: sum over the output columns against x . colsum(W)
    colsum = oracle.dequant(N.SI_Q4_K, blocks, rows * cols).reshape(rows, cols).sum(axis=0, dtype=np.float64)
    want = xf.astype(np.float64) @ colsum
    got = y.sum(axis=1, dtype=np.float64)
    assert rel_l2(got, want) < 1e-3, rel_l2(got, want)
    w.free()


def test_prefill_gemm_wide_range_activations(ctx):
    """Rows whose |x| spans 1e-7 .. 1e5 (f16 alone would overflow above 65504
    and lose the small values), a row of tiny values only, a row of zeros."""
    import torch
    rows, cols, M = 512, 2048, 130
    blocks = synth_blocks_host(N.SI_Q4_K, rows, cols, 5, 9, N.SYNTH_PLAIN, 0.01)
    rng = np.random.default_rng(17)
    mag = 10.0 ** rng.uniform(-7, 5, (M, cols))
    x = mag * rng.choice([-1.0, 1.0], (M, cols))
    x[3] = 1e-7 * rng.standard_normal(cols)   # tiny only
    x[4] = 0.0                                # zeros
    x[5] = 1e5 * rng.standard_normal(cols)    # large only
    xb, xf = bf16_round(x)
    w = ctx.upload(N.SI_Q4_K, blocks, rows, cols)
    y = ctx.qgemm(w, torch.from_numpy(xb.view(np.int16)).cuda().view(torch.bfloat16)).cpu().numpy()
    ctx.synchronize()
    ref = oracle.qmatvec(N.SI_Q4_K, blocks, rows, cols, xf)
    assert np.all(np.isfinite(y))
    assert np.array_equal(y[4], np.zeros(rows, np.float32))
    for m in range(M):
        if m == 4:
            continue
        assert rel_l2(y[m], ref[m]) < 1e-3, (m, rel_l2(y[m], ref[m]))
    w.free()


def test_prefill_attention_2048_causal_32_8_heads(ctx):
    import torch
    S, H, Hkv = 2048, 32, 8
    rng = np.random.default_rng(2048)
    qh, qf = bf16_round(rng.standard_normal((1, H, S, 128)))
    kh, kf = bf16_round(rng.standard_normal((1, Hkv, S, 128)))
    vh, vf = bf16_round(rng.standard_normal((1, Hkv, S, 128)))
    scale = 1.0 / np.sqrt(128.0)
    t = lambda a: torch.from_numpy(a.view(np.int16)).cuda().view(torch.bfloat16)
    out = ctx.attn_prefill(t(qh), t(kh), t(vh), scale, True).cpu().numpy()
    G = H // Hkv
    for h in (0, 5, 18, 31):
        ref = oracle.flash_attention(qf[0, h], kf[0, h // G], vf[0, h // G], scale, True, start_pos=0)
        assert rel_l2(out[0, h], ref) < 1e-4, (h, rel_l2(out[0, h], ref))


def f16_to_f32(a):
    return np.asarray(a, np.uint16).view(np.float16).astype(np.float32)


@pytest.mark.parametrize("pos", [8191, 5000])
def test_decode_attention_ctx8192_70b_heads(ctx, pos):
    import torch
    cfg = config(1, 8192, 1024, 64, 8, 1000, 8192, 1)
    m = DecodeModel(ctx, cfg)
    m.synth(3)
    m.kv_synth(pos, 3)
    nh, nkv, hd = 64, 8, 128
    rng = np.random.default_rng(pos)
    qkv = rng.standard_normal((1, (nh + 2 * nkv) * hd)).astype(np.float32)
    out = m.attention(0, torch.from_numpy(qkv).cuda(), pos).cpu().numpy()
    q, k = oracle.rope_apply(qkv[0, :nh * hd], qkv[0, nh * hd:(nh + nkv) * hd], pos, hd, cfg.rope_theta)
    v = qkv[0, (nh + nkv) * hd:]
    kp, vp = host_kv(cfg, 3, 0, 0, pos)
    K = np.concatenate([f16_to_f32(kp), k.astype(np.float16).astype(np.float32)])
    V = np.concatenate([f16_to_f32(vp), v.astype(np.float16).astype(np.float32)])
    ref = oracle.attention_decode(q, K, V, nh, nkv, hd)
    assert rel_l2(out[0], ref) < 1e-5, rel_l2(out[0], ref)
    m.free()


def q8_row(hidden, rng):
    """One Q8_0 row (hidden / 32 blocks): f16 d > 0, int8 codes in -127..127."""
    nb = hidden // 32
    d = np.full(nb, 0.01 / np.sqrt(hidden), np.float16).view(np.uint8).reshape(nb, 2)
    q = rng.integers(-127, 128, (nb, 32)).astype(np.int8)
    return d, q


def tie_lm_head(vocab, hidden, ties, rng):
    """Q8_0 lm_head whose rows in `ties` equal w and every other row is -w
    (exact negation), so logit[t] = L for t in ties and -L elsewhere."""
    d, q = q8_row(hidden, rng)
    nb = hidden // 32
    pos_row = np.concatenate([d, q.view(np.uint8)], axis=1).reshape(-1)
    neg_row = np.concatenate([d, (-q).astype(np.int8).view(np.uint8)], axis=1).reshape(-1)
    W = np.tile(neg_row, (vocab, 1))
    for t in ties:
        W[t] = pos_row
    return np.ascontiguousarray(W.reshape(vocab, nb * 34))


def test_argmax_ties_take_the_first_index(ctx):
    """Rows 37 and 357 tie at L, every other row at -L: the greedy token is
    37 when L > 0 and 0 otherwise -- the first index of the maximum."""
    vocab, hidden = 1000, 512
    cfg = config(2, hidden, 1024, 4, 2, vocab, 96, 1, lm_head_qtype=N.SI_Q8_0)
    rng = np.random.default_rng(4)
    ties = (37, 357)  # same row inside their 16-row tiles
    W = tie_lm_head(vocab, hidden, ties, rng)
    m = DecodeModel(ctx, cfg)
    m.synth(21)
    m.set_tensor(-1, N.T_LM_HEAD, W)
    m.kv_synth(16, 21)
    om = oracle.synthetic_model(cfg, 21, n_seq=1, kv_len=16)
    om.set(-1, 1, N.SI_Q8_0, W)
    tok, seen = 11, set()
    for s in range(8):
        out, lg = m.step([tok], 16 + s, logits=True)
        L = lg[0, ties[0]]
        assert lg[0, ties[1]] == L
        others = np.delete(lg[0], ties)
        assert np.all(others == -L)
        want = ties[0] if L > 0 else 0
        assert out[0] == want, (s, out[0], L)
        ref = om.forward(0, tok, 16 + s)
        if abs(ref[ties[0]]) > 1e-3 * np.abs(ref).max():
            assert oracle.argmax(ref) == want
        seen.add(want)
        tok = int(out[0])
    m.free()


def test_argmax_all_equal_logits_give_zero(ctx):
    vocab, hidden = 1000, 512
    cfg = config(1, hidden, 1024, 4, 2, vocab, 64, 1, lm_head_qtype=N.SI_Q8_0)
    rng = np.random.default_rng(5)
    W = tie_lm_head(vocab, hidden, range(vocab), rng)  # every row is w
    m = DecodeModel(ctx, cfg)
    m.synth(22)
    m.set_tensor(-1, N.T_LM_HEAD, W)
    m.kv_synth(8, 22)
    out, lg = m.step([3], 8, logits=True)
    assert np.all(lg[0] == lg[0, 0]) and out[0] == 0
    m.free()
