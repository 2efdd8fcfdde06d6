"""The KDA kernels' CPU restatement (oracle: orc_kda_step,
orc_short_conv_step, orc_rmsnorm_gated) against the reference's own
outputs (tests/golden/kda.npz, written by src/kda.c:26-111 compiled from
the reference), bit for bit, over several chained decode steps."""
import numpy as np
import pytest

import oracle as O
from golden_cases import (CONV_C, CONV_KS, KDA_CASES, NORM_DIM, NORM_HEADS, bits, conv_inputs,
                          kda_inputs, load, norm_inputs, sha)


@pytest.mark.parametrize("name", list(KDA_CASES))
def test_kda_step_golden(name):
    g = load("kda")
    H, K, V, T = KDA_CASES[name]
    S = np.zeros((H, K, V), np.float32)
    for t, (q, k, v, gl, beta) in enumerate(kda_inputs(name)):
        S, o = O.kda_step(H, K, V, q, k, v, gl, beta, S)
        assert np.array_equal(bits(o), bits(g[f"{name}_o{t}"]))
    assert sha(S) == str(g[f"{name}_S_sha"])


def test_short_conv_golden():
    g = load("kda")
    w, xs = conv_inputs()
    ring = np.zeros((CONV_C, CONV_KS - 1), np.float32)
    for t in range(xs.shape[0]):
        ring, y = O.short_conv_step(CONV_C, CONV_KS, w, None, ring, xs[t])
        assert np.array_equal(bits(y), bits(g[f"conv_y{t}"]))
    assert np.array_equal(bits(ring), bits(g["conv_ring"]))


def test_rmsnorm_gated_golden():
    g = load("kda")
    x, gate, w, eps = norm_inputs()
    y = np.concatenate([O.rmsnorm_gated(NORM_DIM, x[h * NORM_DIM:(h + 1) * NORM_DIM],
                                        gate[h * NORM_DIM:(h + 1) * NORM_DIM], w, float(eps))
                        for h in range(NORM_HEADS)])
    assert np.array_equal(bits(y), bits(g["norm_y"]))
