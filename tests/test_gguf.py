"""The GGUF reader (si_gguf_*) on files written by gguf-py: header, metadata,
tensor table and bytes, the derived model configuration, and rejection of
malformed or unsupported files.  Host-only: no GPU is used."""
import numpy as np
import pytest

from gguf_util import write_llama_gguf
from sharpinfer_b200 import native as N
from sharpinfer_b200.gguf import GGUFFile
from sharpinfer_b200.model import config


@pytest.fixture(scope="module")
def small(tmp_path_factory):
    cfg = config(2, 512, 1024, 8, 2, 1000, 256, 1)
    path = tmp_path_factory.mktemp("gguf") / "small.gguf"
    written = write_llama_gguf(path, cfg, 7)
    return cfg, path, written


def test_header_metadata_and_tensor_table(small):
    cfg, path, written = small
    with GGUFFile(path) as f:
        version, nt, nkv, off = f.info()
        assert version == 3 and nt == 2 * 9 + 3 and off % 32 == 0
        assert f.meta_string("general.architecture") == "llama"
        assert f.meta_string("general.name") == "synthetic-llama"
        assert f.meta_int("llama.block_count") == 2
        assert f.meta_int("llama.attention.head_count_kv") == 2
        assert abs(f.meta_float("llama.rope.freq_base") - 500000.0) < 1e-3
        with pytest.raises(N.SIError):
            f.meta_int("llama.no_such_key")
        names = {t[0]: t for t in f.tensors()}
        assert names["blk.0.attn_q.weight"][1:4] == (N.SI_Q4_K, 1024, 512)
        assert names["blk.1.ffn_down.weight"][1:4] == (N.SI_Q4_K, 512, 1024)
        assert names["output.weight"][1:4] == (N.SI_Q6_K, 1000, 512)
        assert names["blk.0.attn_norm.weight"][1:4] == (0, 1, 512)
        for name in ("blk.0.attn_q.weight", "blk.1.ffn_up.weight", "output.weight", "output_norm.weight"):
            assert f.tensor_bytes(name) == written[name], name


def test_model_config_from_metadata(small):
    cfg, path, _ = small
    with GGUFFile(path) as f:
        c = f.model_config(max_seq=300, max_batch=2)
    for field in ("n_layers", "hidden", "intermediate", "n_heads", "n_kv_heads", "head_dim", "vocab",
                  "weight_qtype", "lm_head_qtype", "emb_qtype"):
        assert getattr(c, field) == getattr(cfg, field), field
    assert c.max_seq == 300 and c.max_batch == 2
    assert abs(c.rms_eps - 1e-5) < 1e-9 and c.rope_theta == 500000.0


def test_tied_embeddings_and_file_context(tmp_path):
    cfg = config(1, 512, 1024, 4, 2, 1000, 128, 1)
    path = tmp_path / "tied.gguf"
    write_llama_gguf(path, cfg, 3, tied=True)
    with GGUFFile(path) as f:
        c = f.model_config()
    assert c.lm_head_qtype == c.emb_qtype == N.SI_Q4_K and c.max_seq == 128


def test_mixed_projection_types_are_rejected(tmp_path):
    import oracle
    cfg = config(1, 512, 1024, 4, 2, 1000, 128, 1)
    path = tmp_path / "mixed.gguf"
    v6 = oracle.synth_blocks(oracle.Q6_K, 256, 512, 1, 2, 0, 0.01)
    write_llama_gguf(path, cfg, 3, override={(0, 2): (oracle.Q6_K, v6)})
    with GGUFFile(path) as f:
        with pytest.raises(N.SIError) as ei:
            f.model_config()
    assert ei.value.status == 4 and "attn_v" in str(ei.value)


def test_malformed_files_are_rejected(tmp_path, small):
    _, path, _ = small
    data = open(path, "rb").read()
    for name, blob in (("magic", b"GGUX" + data[4:]), ("truncated", data[:200]),
                       ("version", data[:4] + (9).to_bytes(4, "little") + data[8:])):
        p = tmp_path / (name + ".gguf")
        p.write_bytes(blob)
        with pytest.raises(N.SIError):
            GGUFFile(p)
    with pytest.raises(N.SIError):
        GGUFFile(tmp_path / "missing.gguf")
