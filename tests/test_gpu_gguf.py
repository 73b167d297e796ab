"""A model loaded from a GGUF file (si_gguf_model_config + si_model_load_gguf)
decodes exactly like the same weights generated on the device, and like the
oracle's forward pass over the file's tensors (Transformer.Forward,
src/SharpInfer.Core/Layers/Transformer.cs:67-162)."""
import numpy as np
import pytest

import oracle
from conftest import rel_l2
from gguf_util import write_llama_gguf
from sharpinfer_b200.gguf import GGUFFile
from sharpinfer_b200.model import DecodeModel, config

pytestmark = pytest.mark.gpu


def test_gguf_model_decodes_like_the_synthetic_model(ctx, tmp_path):
    cfg = config(2, 1024, 1024, 8, 2, 1000, 128, 1)
    path = tmp_path / "m.gguf"
    write_llama_gguf(path, cfg, 7)
    with GGUFFile(path) as f:
        fc = f.model_config(max_seq=128)
        a = DecodeModel(ctx, fc)
        f.load_into(a)
    b = DecodeModel(ctx, cfg)
    b.synth(7)
    for m in (a, b):
        m.kv_synth(16, 7)
    om = oracle.synthetic_model(cfg, 7, n_seq=1, kv_len=16)
    tok = 5
    for s in range(3):
        oa, la = a.step([tok], 16 + s, logits=True)
        ob, lb = b.step([tok], 16 + s, logits=True)
        assert np.array_equal(la, lb) and oa[0] == ob[0]
        assert rel_l2(la[0], om.forward(0, tok, 16 + s)) < 1e-3
        tok = int(oa[0])
    a.free()
    b.free()


def test_gguf_tied_embeddings(ctx, tmp_path):
    cfg = config(1, 512, 1024, 4, 2, 1000, 64, 1)
    path = tmp_path / "tied.gguf"
    written = write_llama_gguf(path, cfg, 9, tied=True)
    with GGUFFile(path) as f:
        fc = f.model_config()
        m = DecodeModel(ctx, fc)
        f.load_into(m)
    m.kv_synth(8, 9)
    om = oracle.synthetic_model(cfg, 9, n_seq=1, kv_len=8)
    emb = np.frombuffer(written["token_embd.weight"], np.uint8)
    om.set(-1, 1, cfg.emb_qtype, emb)  # lm_head = the embedding rows
    out, lg = m.step([3], 8, logits=True)
    assert rel_l2(lg[0], om.forward(0, 3, 8)) < 1e-3
    m.free()
