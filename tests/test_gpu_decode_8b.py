"""Full-size parity: Llama-3-8B-architecture Q4_K_M greedy decode on the GPU
against 64 tokens the CPU oracle decoded (tests/golden/decode_8b.json, made by
tests/golden/make_decode_golden.py with the reference forward pass,
Transformer.Forward, src/SharpInfer.Core/Layers/Transformer.cs:67-162).

Same seeded weights (Q4_K projections and embedding, Q6_K lm_head) and the same
4096-position f16 KV prefix on both sides; the device run must emit the
identical 64 greedy tokens, and its top-1 logits must match the oracle's.
"""
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN
from sharpinfer_b200.model import DecodeModel, llama3_8b

pytestmark = pytest.mark.gpu
GOLD = os.path.join(GOLDEN, "decode_8b.json")


@pytest.fixture(scope="module")
def gold():
    return json.load(open(GOLD))


@pytest.fixture(scope="module")
def model8b(ctx, gold):
    cfg = llama3_8b(max_seq=gold["kv_len"] + gold["steps"] + 8)
    for f, v in gold["config"].items():
        if f not in ("max_seq",):
            assert getattr(cfg, f) == pytest.approx(v), f
    m = DecodeModel(ctx, cfg)
    m.synth(gold["seed"])
    yield m
    m.free()


def test_8b_greedy_tokens_match_oracle(model8b, gold):
    m = model8b
    m.kv_synth(gold["kv_len"], gold["seed"])
    gen = m.generate([gold["start_token"]], gold["kv_len"], gold["steps"])[:, 0]
    first_bad = next((i for i, (a, b) in enumerate(zip(gen, gold["tokens"])) if a != b), None)
    assert first_bad is None, (first_bad, gold["records"][first_bad] if first_bad is not None else None)


def test_8b_logits_track_oracle(model8b, gold):
    """Per-step top-1 logit and top-1/top-2 margin against the oracle's, host-driven steps."""
    m = model8b
    m.kv_synth(gold["kv_len"], gold["seed"])
    for r in gold["records"][:8]:
        out, lg = m.step([r["input"]], r["pos"], logits=True)
        top = np.sort(lg[0])[-2:]
        assert int(out[0]) == r["token"], r
        assert abs(top[1] - r["top1"]) <= 1e-3 * max(1.0, abs(r["top1"])), (r, top)
        assert abs((top[1] - top[0]) - r["margin"]) <= 2e-3 * max(1.0, abs(r["top1"])), (r, top)
