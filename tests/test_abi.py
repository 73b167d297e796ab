"""The C-ABI library loads and exports what include/sharpinfer_b200.h declares (no GPU)."""
import ctypes
import os

import numpy as np
import pytest

from conftest import ROOT
from sharpinfer_b200 import native as N
from sharpinfer_b200.backend import synth_blocks_host, synth_f16_host, synth_f32_host


def test_library_exports_every_declared_symbol():
    lib = N.load()
    names = N.declared_symbols()
    assert len(names) >= 15
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert set(names) <= set(N._SIGS) | set(getattr(N, "_LEGACY_SIGS", {})), "binding lacks signatures"


def test_version():
    assert N.load().si_version() >= 100


def test_init_reports_errors_without_crashing():
    import torch
    h = ctypes.c_void_p()
    if torch.cuda.is_available():
        st = N.load().si_init(10_000, ctypes.byref(h))
        assert st == 1 and b"out of range" in N.load().si_last_error()
    else:
        st = N.load().si_init(0, ctypes.byref(h))
        assert st == 2 and h.value is None
        assert len(N.load().si_last_error()) > 0


def test_null_arguments_are_rejected():
    lib = N.load()
    assert lib.si_qmatvec(None, None, None, None, 1) == 1
    assert b"NULL" in lib.si_last_error()
    assert lib.si_synth_blocks_host(99, 1, 256, 0, 0, 0, 0.01, None) == 1


def test_host_generator_is_deterministic_and_seeded():
    a = synth_blocks_host(N.SI_Q4_K, 4, 512, 42, 1)
    b = synth_blocks_host(N.SI_Q4_K, 4, 512, 42, 1)
    c = synth_blocks_host(N.SI_Q4_K, 4, 512, 43, 1)
    assert np.array_equal(a, b) and not np.array_equal(a, c)
    x = synth_f32_host(100000, 5, 6)
    assert abs(x.mean()) < 0.02 and abs(x.std() - 1) < 0.02
    h = synth_f16_host(1000, 5, 7).view(np.float16).astype(np.float32)
    assert abs(h.std() - 1) < 0.1


def test_model_recipe_is_zero_mean():
    """SI_SYNTH_MODEL Q4_K blocks: dmin == d and m = round(7.5 sc), so weights average ~0."""
    import oracle
    blocks = synth_blocks_host(N.SI_Q4_K, 64, 1024, 11, 3, N.SYNTH_MODEL, 0.01).reshape(-1, 144)
    assert np.array_equal(blocks[:, 0:2], blocks[:, 2:4])
    W = oracle.dequant(N.SI_Q4_K, blocks.ravel(), 64 * 1024)
    assert abs(W.mean()) < 0.05 * W.std()


@pytest.mark.parametrize("qt,rows,cols", [(N.SI_Q4_K, 3, 100), (7, 1, 256)])
def test_host_generator_rejects_bad_shapes(qt, rows, cols):
    with pytest.raises(N.SIError):
        synth_blocks_host(qt, rows, cols, 1, 1)


def test_csharp_binding_names_exist_in_the_library():
    """Every function the C# backend (sharpinfer_b200/csharp/B200Backend.cs)
    imports is declared in the header and exported, with as many parameters
    as the header gives it; its config struct has si_model_config's fields."""
    import re
    src = open(os.path.join(ROOT, "sharpinfer_b200", "csharp", "B200Backend.cs")).read()
    header = open(N.HEADER).read()
    imports = re.findall(r"public static extern \w+\*? (\w+)\(([^)]*)\);", src)
    assert len(imports) >= 20
    lib = N.load()
    for name, params in imports:
        assert hasattr(lib, name), name
        m = re.search(r"SI_EXPORT[^;(]*\b%s\s*\(([^)]*)\)" % name, header)
        assert m, name
        n_h = 0 if m.group(1).strip() in ("", "void") else m.group(1).count(",") + 1
        n_c = 0 if not params.strip() else params.count(",") + 1
        assert n_h == n_c, (name, n_h, n_c)
    struct = re.search(r"public struct B200ModelConfig\s*\{(.*?)\}", src, re.S).group(1)
    fields = sum(line.count(",") + 1 for line in struct.split(";") if line.strip().startswith("public"))
    assert fields == len(N.ModelConfig._fields_)
