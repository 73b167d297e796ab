"""The oracle and the library generate the seeded synthetic model from one
input generator (sharpinfer_b200/csrc/synth.h), each in its own build: the
oracle's copy lets the timed CPU baseline run without loading the library
under test.  These CPU tests check that both builds give the same bytes and
that the oracle's tensor table matches the library's si_model_tensor_recipe
for the 8B and 70B architectures (every tag, type, scale and shape)."""
import numpy as np
import pytest

import oracle
from sharpinfer_b200 import native as N
from sharpinfer_b200.backend import synth_blocks_host, synth_f16_host, synth_f32_host
from sharpinfer_b200.model import llama3_70b, llama3_8b, tensor_recipe


@pytest.mark.parametrize("qt,recipe,sigma", [(N.SI_Q4_K, N.SYNTH_MODEL, 1.0 / (23.3 * 64)),
                                             (N.SI_Q4_K, N.SYNTH_PLAIN, 0.01),
                                             (N.SI_Q6_K, N.SYNTH_PLAIN, 1.0 / (348 * 64)),
                                             (N.SI_Q8_0, N.SYNTH_PLAIN, 1.0 / (73.9 * 64))])
def test_oracle_blocks_equal_library_blocks(qt, recipe, sigma):
    a = oracle.synth_blocks(qt, 48, 1024, 77, 1003, recipe, sigma)
    b = synth_blocks_host(qt, 48, 1024, 77, 1003, recipe, sigma)
    assert np.array_equal(a, np.asarray(b).view(np.uint8).ravel())


def test_oracle_vectors_equal_library_vectors():
    assert np.array_equal(oracle.synth_f32(5000, 3, 9, 1.0, 0.01).view(np.uint32),
                          np.asarray(synth_f32_host(5000, 3, 9, 1.0, 0.01)).view(np.uint32))
    lib = N.load()
    tag = lib.si_model_kv_tag(7, 3, 1)
    assert tag == oracle.kv_tag(7, 3, 1)
    assert np.array_equal(oracle.synth_f16(7000, 3, tag), np.asarray(synth_f16_host(7000, 3, tag)).view(np.uint16))


@pytest.mark.parametrize("make", [llama3_8b, llama3_70b])
def test_oracle_recipe_table_equals_library(make):
    cfg = make()
    items = [(l, t) for l in (0, 1, cfg.n_layers - 1) for t in range(9)]
    items += [(-1, t) for t in (N.T_EMB, N.T_LM_HEAD, N.T_FINAL_NORM)]
    for layer, t in items:
        a = oracle.tensor_recipe(cfg, layer, t)
        b = tensor_recipe(cfg, layer, t)
        assert a[:3] == b[:3] and a[5:] == b[5:], (layer, t, a, b)
        assert np.float32(a[3]) == np.float32(b[3]) and np.float32(a[4]) == np.float32(b[4]), (layer, t, a, b)
