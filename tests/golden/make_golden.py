"""Generate the dequantisation golden vectors in tests/golden/dequant.npz.

The expected values come from gguf-py (the GGML project's reference Python
implementation of the Q4_K / Q6_K / Q8_0 block formats, version recorded in
the file), which performs the same f32 operations in the same order as
SharpInfer's Dequantize class (src/SharpInfer.Core/Tensors/Quantization.cs:
Q4_K :273-314 (d*sc)*q - dmin*m, Q6_K :362-391 (d*sc)*(q-32), Q8_0 :106-114
q*d).  The inputs are seeded synthetic blocks (the library's host generator)
plus hand-built edge blocks: both GetScaleMinK4 branches, extreme scales,
signed zero, subnormal, negative, infinite and NaN block scales.

Run from the repository root:  python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import gguf  # noqa: E402
from gguf import quants  # noqa: E402

from sharpinfer_b200 import native as N  # noqa: E402
from sharpinfer_b200.backend import synth_blocks_host  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "dequant.npz")
GT = {N.SI_Q4_K: gguf.GGMLQuantizationType.Q4_K, N.SI_Q6_K: gguf.GGMLQuantizationType.Q6_K,
      N.SI_Q8_0: gguf.GGMLQuantizationType.Q8_0}


def f16bits(x):
    return int(np.array([x], np.float16).view(np.uint16)[0])


def put16(b, off, v):
    b[off] = v & 0xFF
    b[off + 1] = v >> 8


def edge_q4k():
    blocks = []
    heads = [(0x3C00, 0x3800), (0xBC00, 0x3C00), (0x0001, 0x03FF), (0x8000, 0x0000),
             (0x7BFF, 0x7BFF), (0x7C00, 0x3C00), (0x3C00, 0x7E00), (f16bits(0.0123), f16bits(0.00456))]
    rng = np.random.default_rng(7)
    for i, (d, dm) in enumerate(heads):
        b = np.zeros(144, np.uint8)
        put16(b, 0, d)
        put16(b, 2, dm)
        if i == 0:  # top bits set in every byte: exercises both GetScaleMinK4 branches
            b[4:16] = [0xC1, 0x42, 0x83, 0x04, 0x45, 0x86, 0xC7, 0x08, 0x9A, 0xBC, 0xDE, 0xF1]
        elif i == 1:
            b[4:16] = 0xFF
        else:
            b[4:16] = rng.integers(0, 256, 12)
        b[16:] = (np.arange(128) * 37 + i) & 0xFF
        blocks.append(b)
    return np.concatenate(blocks)


def edge_q6k():
    blocks = []
    rng = np.random.default_rng(8)
    ds = [0x3C00, 0xB800, 0x0001, 0x7BFF, 0x7C00, 0x7E00, f16bits(3.1e-5), 0x0000]
    for i, d in enumerate(ds):
        b = np.zeros(210, np.uint8)
        b[:128] = (np.arange(128) * 29 + 3 * i) & 0xFF
        b[128:192] = (np.arange(64) * 53 + i) & 0xFF
        sc = np.array([-128, 127, 0, 1, -1, 32, -32, 5, -7, 64, -64, 100, -100, 2, -2, 3], np.int8)
        b[192:208] = np.roll(sc, i).view(np.uint8) if i < 4 else rng.integers(0, 256, 16)
        put16(b, 208, d)
        blocks.append(b)
    return np.concatenate(blocks)


def edge_q80():
    blocks = []
    ds = [0x3C00, 0xBC00, 0x0001, 0x7BFF, 0x7C00, 0x7E00, 0x8000, f16bits(0.0071)]
    for i, d in enumerate(ds):
        b = np.zeros(34, np.uint8)
        put16(b, 0, d)
        b[2:] = ((np.arange(32) * 8 + 128 + i) & 0xFF)  # spans -128..127
        blocks.append(b)
    return np.concatenate(blocks)


def canon_bits(a):
    """f32 bit patterns with every NaN mapped to 0x7FC00000."""
    a = np.asarray(a, np.float32).copy()
    bits = a.view(np.uint32).copy()
    bits[np.isnan(a)] = 0x7FC00000
    return bits


def main():
    cases = {
        # name: (qtype, rows, cols, blocks)
        "q4k_plain": (N.SI_Q4_K, 24, 512, synth_blocks_host(N.SI_Q4_K, 24, 512, 1234, 1, N.SYNTH_PLAIN, 0.01)),
        "q4k_model": (N.SI_Q4_K, 16, 256, synth_blocks_host(N.SI_Q4_K, 16, 256, 1234, 2, N.SYNTH_MODEL, 0.002)),
        "q4k_edge": (N.SI_Q4_K, 8, 256, edge_q4k()),
        "q6k_plain": (N.SI_Q6_K, 20, 512, synth_blocks_host(N.SI_Q6_K, 20, 512, 1234, 3, N.SYNTH_PLAIN, 0.01)),
        "q6k_edge": (N.SI_Q6_K, 8, 256, edge_q6k()),
        "q80_plain": (N.SI_Q8_0, 18, 256, synth_blocks_host(N.SI_Q8_0, 18, 256, 1234, 4, N.SYNTH_PLAIN, 0.01)),
        "q80_edge": (N.SI_Q8_0, 8, 32, edge_q80()),
    }
    arrays = {"gguf_version": np.array(gguf.__version__ if hasattr(gguf, "__version__") else
                                       __import__("importlib.metadata").metadata.version("gguf"))}
    for name, (qt, rows, cols, blocks) in cases.items():
        bb = N.BLOCK_BYTES[qt]
        with np.errstate(all="ignore"):
            ref = quants.dequantize(blocks.reshape(-1, bb), GT[qt]).astype(np.float32).reshape(rows, cols)
        arrays[name + "_meta"] = np.array([qt, rows, cols], np.int64)
        arrays[name + "_blocks"] = blocks
        arrays[name + "_bits"] = canon_bits(ref)
    np.savez_compressed(OUT, **arrays)
    print("wrote", OUT, {k: v.shape for k, v in arrays.items()})


if __name__ == "__main__":
    main()
