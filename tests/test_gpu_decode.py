"""GPU parity of attention decode and the full decode step through the C ABI.

The oracle is the reference forward pass (Transformer.Forward,
src/SharpInfer.Core/Layers/Transformer.cs:67-162) restated in oracle.cpp, fed
the same seeded weights and KV prefix on the host.  Its KV cache rounds newly
stored K/V through f16 (the device cache is f16; the reference's is f32).
Logits must agree within 1e-3 relative L2 (checked much tighter) and greedy
tokens must be identical.
"""
import numpy as np
import pytest

import oracle
from conftest import rel_l2
from sharpinfer_b200 import native as N
from sharpinfer_b200.model import DecodeModel, config, host_kv

pytestmark = pytest.mark.gpu
SEED = 7


def small_cfg(G, layers=2, max_batch=2, max_seq=320, qt=N.SI_Q4_K, vocab=1000, inter=768):
    nkv = 2
    nh = nkv * G
    return config(layers, nh * 128, inter, nh, nkv, vocab, max_seq, max_batch, weight_qtype=qt)


def f16_to_f32(a):
    return np.asarray(a, np.uint16).view(np.float16).astype(np.float32)


@pytest.mark.parametrize("G", [1, 2, 4, 8])
@pytest.mark.parametrize("pos", [0, 1, 63, 64, 65, 129, 300, 319])
def test_attention_layer_matches_oracle(ctx, G, pos):
    import torch
    cfg = small_cfg(G, layers=1)
    m = DecodeModel(ctx, cfg)
    m.synth(SEED)
    m.kv_synth(pos, SEED)  # positions [0, pos) prefilled; pos is appended by the kernel
    nh, nkv, hd = cfg.n_heads, cfg.n_kv_heads, 128
    B = 2
    rng = np.random.default_rng(pos * 10 + G)
    qkv = rng.standard_normal((B, (nh + 2 * nkv) * hd)).astype(np.float32)
    out = m.attention(0, torch.from_numpy(qkv).cuda(), pos).cpu().numpy()
    for b in range(B):
        q, k = oracle.rope_apply(qkv[b, :nh * hd], qkv[b, nh * hd:(nh + nkv) * hd], pos, hd, cfg.rope_theta)
        v = qkv[b, (nh + nkv) * hd:]
        kp, vp = host_kv(cfg, SEED, 0, b, pos)
        K = np.concatenate([f16_to_f32(kp), k.astype(np.float16).astype(np.float32)])
        V = np.concatenate([f16_to_f32(vp), v.astype(np.float16).astype(np.float32)])
        ref = oracle.attention_decode(q, K, V, nh, nkv, hd)
        assert rel_l2(out[b], ref) < 1e-5, (b, rel_l2(out[b], ref))
    m.free()


def run_parity(ctx, cfg, kv_len, steps, start_tokens):
    m = DecodeModel(ctx, cfg)
    m.synth(SEED)
    m.kv_synth(kv_len, SEED)
    B = len(start_tokens)
    om = oracle.synthetic_model(cfg, SEED, n_seq=B, kv_len=kv_len)
    toks = list(start_tokens)
    worst = 0.0
    for s in range(steps):
        pos = kv_len + s
        out, lg = m.step(toks, pos, logits=True)
        nxt = []
        for b in range(B):
            ref = om.forward(b, toks[b], pos)
            err = rel_l2(lg[b], ref)
            worst = max(worst, err)
            assert err < 1e-3, (s, b, err)
            top = np.sort(ref)[-2:]
            if top[1] - top[0] > 1e-4 * max(1.0, abs(top[1])):
                assert out[b] == oracle.argmax(ref), (s, b)
            nxt.append(int(out[b]))
        toks = nxt
    m.free()
    return worst


@pytest.mark.parametrize("G", [1, 2, 4, 8])  # G = 1: the splits are merged by k_prep, else in the kernel
def test_decode_steps_match_oracle(ctx, G):
    worst = run_parity(ctx, small_cfg(G), kv_len=100, steps=5, start_tokens=[5, 777])
    assert worst < 2e-5, worst


@pytest.mark.parametrize("qt", [N.SI_Q6_K, N.SI_Q8_0])
def test_decode_other_weight_types(ctx, qt):
    cfg = small_cfg(4, qt=qt)
    assert run_parity(ctx, cfg, kv_len=40, steps=3, start_tokens=[11]) < 2e-5


def test_decode_from_empty_cache(ctx):
    """pos 0: attention over the single stored position."""
    assert run_parity(ctx, small_cfg(2, layers=1, max_batch=1), kv_len=0, steps=3, start_tokens=[42]) < 2e-5


def test_decode_batch5_uses_two_mma_groups(ctx):
    cfg = small_cfg(2, layers=1, max_batch=5)
    assert run_parity(ctx, cfg, kv_len=64, steps=2, start_tokens=[1, 2, 3, 4, 999]) < 2e-5


def test_batch_rows_are_independent(ctx):
    """Sequence b of a batch equals the same sequence decoded alone (batch 1
    runs its own matvec kernel, so the summation order differs slightly)."""
    cfg = small_cfg(4, max_batch=2)
    m = DecodeModel(ctx, cfg)
    m.synth(SEED)
    m.kv_synth(50, SEED)
    _, lg2 = m.step([9, 9], 50, logits=True)
    m.kv_synth(50, SEED)
    _, lg1 = m.step([9], 50, logits=True)
    assert rel_l2(lg2[0], lg1[0]) < 1e-5
    m.free()


def test_step_rejects_bad_arguments(ctx):
    cfg = small_cfg(2, layers=1, max_batch=1, max_seq=64)
    m = DecodeModel(ctx, cfg)
    m.synth(SEED)
    with pytest.raises(N.SIError):
        m.step([1], 64)  # pos == max_seq (KVCache.Store throws, KVCache.cs:48-49)
    with pytest.raises(N.SIError):
        m.step([1000], 0)  # token outside the vocabulary
    with pytest.raises(N.SIError):
        m.step([1, 2], 0)  # batch above max_batch
    m.free()


def test_generate_matches_stepping(ctx):
    """The device-resident loop (si_decode_generate) equals host-driven steps and the oracle."""
    cfg = small_cfg(4, layers=2, max_batch=2)
    m = DecodeModel(ctx, cfg)
    m.synth(SEED)
    m.kv_synth(30, SEED)
    gen = m.generate([3, 500], 30, 6)
    m.kv_synth(30, SEED)
    toks = [3, 500]
    stepped = []
    for s in range(6):
        toks = list(m.step(toks, 30 + s))
        stepped.append(toks)
    assert np.array_equal(gen, np.array(stepped))
    om = oracle.synthetic_model(cfg, SEED, n_seq=2, kv_len=30)
    for b, t0 in enumerate([3, 500]):
        tok = t0
        for s in range(6):
            tok = oracle.argmax(om.forward(b, tok, 30 + s))
            assert tok == gen[s, b]
    m.free()


def test_decode_70b_shapes_batch16_ctx8192(ctx):
    """Llama-3-70B layer shapes (hidden 8192, 64/8 heads, FFN 28672, vocab
    128256) cut to one layer, 16 sequences each with its own 8192-position
    KV prefix, two greedy steps: the batch-16 path of every kernel (the
    tensor-core Q4_K matvec, batch attention, Q6_K lm_head) against the
    oracle per sequence."""
    cfg = config(1, 8192, 28672, 64, 8, 128256, 8200, 16)
    starts = [(128000 + 7919 * b) % 128256 for b in range(16)]
    worst = run_parity(ctx, cfg, kv_len=8192, steps=2, start_tokens=starts)
    assert worst < 2e-5, worst
