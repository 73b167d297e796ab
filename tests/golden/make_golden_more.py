"""Generate tests/golden/dequant_more.npz: golden vectors for the Q4_0, Q2_K,
Q3_K and Q5_K block formats.

The expected values come from gguf-py (the GGML project's Python
implementation of its block formats).  These are the layouts GGUF files hold:
Q2_K [scales 16][qs 64][f16 d][f16 dmin], Q3_K [hmask 32][qs 64][scales 12]
[f16 d], Q5_K [f16 d][f16 dmin][scales 12][qh 32][qs 128], Q4_0 [f16 d][qs 16].
SharpInfer's decoders for Q2_K, Q3_K and Q5_K (src/SharpInfer.Core/Tensors/
Quantization.cs:176-197, :205-267, :322-356) read d, dmin, qh and qs at other
offsets, and Q2_K in another element order; its Q4_0 (:71-83) matches.  The
inputs are seeded random blocks with finite block scales plus edge blocks
(zero, subnormal, negative, infinite and NaN scales).

Run from the repository root:  python tests/golden/make_golden_more.py
"""
import importlib.metadata
import os

import numpy as np
from gguf import GGMLQuantizationType as Q
from gguf import quants

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "dequant_more.npz")
# ggml type id: (gguf-py type, block elements, block bytes, offsets of the f16 scales)
FORMATS = {2: (Q.Q4_0, 32, 18, (0,)), 10: (Q.Q2_K, 256, 84, (80, 82)), 11: (Q.Q3_K, 256, 110, (108,)),
           13: (Q.Q5_K, 256, 176, (0, 2))}
EDGE = [0x3C00, 0xBC00, 0x0001, 0x8000, 0x7BFF, 0x7C00, 0x7E00, 0x2E66]


def blocks_for(qt, nblk, seed, edge):
    _, be, bb, offs = FORMATS[qt]
    rng = np.random.default_rng(seed)
    b = rng.integers(0, 256, (nblk, bb)).astype(np.uint8)
    for i in range(nblk):
        for k, off in enumerate(offs):
            if edge:
                v = EDGE[(i + 3 * k) % len(EDGE)]
            else:
                v = int(np.array([abs(rng.normal()) * 0.01], np.float16).view(np.uint16)[0])
            b[i, off] = v & 0xFF
            b[i, off + 1] = v >> 8
    return b


def canon_bits(a):
    a = np.asarray(a, np.float32).copy()
    bits = a.view(np.uint32).copy()
    bits[np.isnan(a)] = 0x7FC00000
    return bits


def main():
    arrays = {"gguf_version": np.array(importlib.metadata.version("gguf"))}
    for qt, (gt, be, bb, _) in FORMATS.items():
        for name, nblk, edge in (("plain", 64, False), ("edge", 16, True)):
            blk = blocks_for(qt, nblk, 100 + qt, edge)
            with np.errstate(all="ignore"):
                ref = quants.dequantize(blk, gt).astype(np.float32).ravel()
            key = "t%d_%s" % (qt, name)
            arrays[key + "_blocks"] = blk.ravel()
            arrays[key + "_bits"] = canon_bits(ref)
    np.savez_compressed(OUT, **arrays)
    print("wrote", OUT, sorted(arrays))


if __name__ == "__main__":
    main()
