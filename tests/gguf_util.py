"""Writes small llama-architecture GGUF files for the reader tests with
gguf-py (the ggml project's own writer, an implementation independent of
the library's reader): the seeded synthetic model's tensors as raw blocks."""
import numpy as np

import oracle

LAYER_NAMES = ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down", "attn_norm", "ffn_norm")


def write_llama_gguf(path, cfg, seed, tied=False, override=None, version_arch="llama"):
    """The synthetic model of `cfg` as a GGUF v3 file; returns {name: bytes}."""
    from gguf import GGMLQuantizationType as Q
    from gguf import GGUFWriter
    w = GGUFWriter(str(path), version_arch)
    w.add_block_count(cfg.n_layers)
    w.add_embedding_length(cfg.hidden)
    w.add_feed_forward_length(cfg.intermediate)
    w.add_head_count(cfg.n_heads)
    w.add_head_count_kv(cfg.n_kv_heads)
    w.add_key_length(cfg.head_dim)
    w.add_value_length(cfg.head_dim)
    w.add_context_length(cfg.max_seq)
    w.add_layer_norm_rms_eps(cfg.rms_eps)
    w.add_rope_freq_base(cfg.rope_theta)
    w.add_string("general.name", "synthetic-llama")
    qtypes = {12: Q.Q4_K, 14: Q.Q6_K, 8: Q.Q8_0}
    written = {}

    def put(name, data, qt, rows, cols):
        data = np.ascontiguousarray(data)
        if qt == 0:
            arr = data.view(np.float32).reshape(cols)
            w.add_tensor(name, arr)
        else:
            raw = data.view(np.uint8).reshape(rows, -1)
            w.add_tensor(name, raw, raw_dtype=qtypes[qt])
        written[name] = data.view(np.uint8).tobytes()

    for l in range(cfg.n_layers):
        for t, nm in enumerate(LAYER_NAMES):
            tag, qt, rc, sg, mu, rows, cols = oracle.tensor_recipe(cfg, l, t)
            data = oracle.host_tensor(cfg, seed, l, t)
            if override and (l, t) in override:
                qt, data = override[(l, t)]
            put("blk.%d.%s.weight" % (l, nm), data, qt, rows, cols)
    for t, nm in ((oracle.T_EMB, "token_embd"), (oracle.T_LM_HEAD, "output"), (oracle.T_FINAL_NORM, "output_norm")):
        if tied and nm == "output":
            continue
        tag, qt, rc, sg, mu, rows, cols = oracle.tensor_recipe(cfg, -1, t)
        put(nm + ".weight", oracle.host_tensor(cfg, seed, -1, t), qt, rows, cols)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return written
