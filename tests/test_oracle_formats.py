"""Q4_0, Q2_K, Q3_K and Q5_K in the oracle, pinned bit for bit to gguf-py's
decoders (tests/golden/dequant_more.npz, made by make_golden_more.py) -- the
GGML block layouts GGUF files hold.  The reference's own Q2_K / Q3_K / Q5_K
decoders (Quantization.cs:176-197, :205-267, :322-356) read d, dmin, qh and qs
at other offsets (and Q2_K in another element order); the last test shows
that on the same bytes they give different values, while its Q4_0
(Quantization.cs:71-83) agrees."""
import os

import numpy as np
import pytest

import oracle
from conftest import GOLDEN

G = np.load(os.path.join(GOLDEN, "dequant_more.npz"))
BB = {2: (32, 18), 10: (256, 84), 11: (256, 110), 13: (256, 176)}


def canon(a):
    bits = np.asarray(a, np.float32).view(np.uint32).copy()
    bits[np.isnan(a)] = 0x7FC00000
    return bits


@pytest.mark.parametrize("qt", [2, 10, 11, 13])
@pytest.mark.parametrize("case", ["plain", "edge"])
def test_oracle_matches_gguf_py(qt, case):
    blk = G["t%d_%s_blocks" % (qt, case)]
    want = G["t%d_%s_bits" % (qt, case)]
    be, bb = BB[qt]
    got = oracle.dequant(qt, blk, blk.size // bb * be)
    with np.errstate(invalid="ignore"):
        assert np.array_equal(canon(got), want)


@pytest.mark.parametrize("qt", [10, 11, 13])
def test_reference_decoders_read_other_offsets(qt):
    blk = G["t%d_plain_blocks" % qt]
    nb = blk.size // BB[qt][1]
    ref = oracle.dequant_reference_as_written(qt, blk, nb)
    ggml = oracle.dequant(qt, blk, nb * 256)
    with np.errstate(invalid="ignore"):
        assert not np.array_equal(canon(ref), canon(ggml))
