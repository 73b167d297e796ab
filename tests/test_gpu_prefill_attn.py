"""Tensor-core prefill attention (si_attn_prefill) against the oracle's
FlashAttention.Forward restatement (src/SharpInfer.Core/Layers/FlashAttention.cs:59-167),
head by head with the grouped-query mapping h -> h / (H / Hkv).  Inputs are
bf16, so the oracle gets exactly the same values as f32.  Bar: relative L2
1e-4 (probabilities enter the P.V product as bf16 hi + lo, ~16 bits)."""
import numpy as np
import pytest

import oracle
from conftest import rel_l2

pytestmark = pytest.mark.gpu


def bf16(a):
    b = np.ascontiguousarray(a, np.float32).view(np.uint32)
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    return r, (r.astype(np.uint32) << 16).view(np.float32)


@pytest.mark.parametrize("B,H,Hkv,S,KV,causal", [
    (1, 4, 1, 64, 64, True),      # one tile, GQA 4
    (2, 4, 2, 130, 130, True),    # ragged tiles
    (1, 2, 2, 70, 200, True),     # cached prefix: start_pos = KV - S
    (1, 8, 2, 96, 33, False),     # non-causal, KV < one tile
    (1, 2, 1, 256, 256, True),    # key tiles wrap the 3-stage ring
    (1, 4, 1, 200, 520, True),    # two query blocks over 9 key tiles, start_pos 320
    (1, 2, 1, 1, 70, True),       # a single query row
])
def test_prefill_attention_matches_oracle(ctx, B, H, Hkv, S, KV, causal):
    import torch
    rng = np.random.default_rng(S * 7 + KV)
    qh, qf = bf16(rng.standard_normal((B, H, S, 128)))
    kh, kf = bf16(rng.standard_normal((B, Hkv, KV, 128)))
    vh, vf = bf16(rng.standard_normal((B, Hkv, KV, 128)))
    scale = 1.0 / np.sqrt(128.0)
    t = lambda a: torch.from_numpy(a.view(np.int16)).cuda().view(torch.bfloat16)
    out = ctx.attn_prefill(t(qh), t(kh), t(vh), scale, causal).cpu().numpy()
    G = H // Hkv
    for b in range(B):
        for h in range(H):
            ref = oracle.flash_attention(qf[b, h], kf[b, h // G], vf[b, h // G], scale, causal, start_pos=KV - S)
            err = rel_l2(out[b, h], ref)
            assert err < 1e-4, (b, h, err)


def test_prefill_attention_without_keys_is_zero(ctx):
    import torch
    q = torch.ones(1, 2, 5, 128, dtype=torch.bfloat16, device="cuda")
    k = torch.zeros(1, 1, 0, 128, dtype=torch.bfloat16, device="cuda")
    out = ctx.attn_prefill(q, k, k, 0.1, True, start_pos=0)
    assert out.shape == (1, 2, 5, 128) and float(out.abs().max()) == 0.0


def test_prefill_attention_rejects_bad_shapes(ctx):
    import torch
    from sharpinfer_b200 import native as N
    q = torch.zeros(1, 3, 8, 128, dtype=torch.bfloat16, device="cuda")
    k = torch.zeros(1, 2, 8, 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(N.SIError):
        ctx.attn_prefill(q, k, k, 0.1)  # 3 heads over 2 kv heads
