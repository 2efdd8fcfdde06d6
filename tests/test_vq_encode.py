"""The converter's RVQ encoder restated on the CPU (oracle: orc_vq_encode,
orc_vq_lloyd) against the reference's own outputs (tests/golden/enc.npz,
written by src/vq.c:50-136 compiled from the reference), bit for bit:
codes, ties (the first index wins), a dimension other than 8, and one
Lloyd iteration including empty clusters."""
import numpy as np
import pytest

import oracle as O
from golden_cases import ENC_CASES, LLOYD_CASES, bits, enc_inputs, load, lloyd_inputs, sha


@pytest.mark.parametrize("name", list(ENC_CASES))
def test_encode_golden(name):
    g = load("enc")
    X, books = enc_inputs(name)
    assert sha(X, books) == str(g[f"{name}_sha"])
    codes = O.vq_encode(X, books)
    assert np.array_equal(codes, g[f"{name}_codes"])
    if name == "enc_ties":               # a duplicated entry never wins over its first copy
        assert codes.max() < books.shape[1] // 2


@pytest.mark.parametrize("name", list(LLOYD_CASES))
def test_lloyd_golden(name):
    g = load("enc")
    X, C0 = lloyd_inputs(name)
    assert sha(X, C0) == str(g[f"{name}_sha"])
    C, live = O.vq_lloyd(X, C0)
    assert live == int(g[f"{name}_live"])
    assert np.array_equal(bits(C), bits(g[f"{name}_C"]))
