"""The VQ4P format's CPU restatement (oracle/vq3r_oracle.c orc_vq4p_*)
against fixtures written by the reference itself (tests/golden/vq4p.npz,
moe_vq4p*.npz: src/model.c:2026-2229 vq_quant_range / vq_rows_p6 and the
moe_layer / moe_chunk loops over VQ4P banks), bit for bit."""
import numpy as np
import pytest

import oracle as O
from golden_cases import (VQ4P_CASES, VQ4P_MOE_CASES, bits, load, rel_l2, sha, vq4p_books,
                          vq4p_case)
from warp_b200 import synth


def test_unpack_matches_converter_packing():
    """tools/convert.py:315-337: byte0 = s0 | s1<<6, byte1 = s1>>2 | s2<<4,
    byte2 = s2>>4 | s3<<2; unpack_p6 inverts it for every index value."""
    rng = np.random.default_rng(3)
    s = rng.integers(0, 64, size=(1000, 4))
    b = np.stack([(s[:, 0] | (s[:, 1] << 6)) & 0xFF,
                  ((s[:, 1] >> 2) | (s[:, 2] << 4)) & 0xFF,
                  ((s[:, 2] >> 4) | (s[:, 3] << 2)) & 0xFF], axis=1).astype(np.uint8)
    assert np.array_equal(synth.unpack_p6(b), s.astype(np.uint8))


@pytest.mark.parametrize("name", list(VQ4P_CASES))
def test_vq4p_matvec_golden(name):
    g = load("vq4p")
    raw = vq4p_books()
    assert sha(raw) == str(g["books_sha"])
    idx, sc, x, M, N = vq4p_case(name)
    assert sha(idx, sc, x) == str(g[f"{name}_sha"]), "generator drifted from the fixture"
    books = synth.flush_f16(raw)
    cb = int(g["cb_base"])
    y = O.vq4p_matvec(idx, sc, x, M, N, books, cb, fma=1)
    assert np.array_equal(bits(y), bits(g[f"{name}_y"]))
    q, qs = O.vq4p_table(books, cb, x, fma=1)
    assert np.array_equal(q, g[f"{name}_q"])
    assert np.array_equal(bits(qs), bits(g[f"{name}_qs"]))
    if N >= 512:
        assert g[f"{name}_qs"][1] == 0.0 and not g[f"{name}_q"][32:64].any()


def _layer(name):
    from golden.make_golden import layer_sha
    seed, kw, xseed, T = VQ4P_MOE_CASES[name]
    L = synth.moe_layer(seed, **kw)
    g = load(name)
    assert layer_sha(L) == str(g["sha"]), "synthetic generator drifted from the fixture"
    return L, synth.activations(xseed, L.hidden, T=max(T, 2)), g, T


@pytest.mark.parametrize("name", list(VQ4P_MOE_CASES))
def test_vq4p_moe_layer_golden(name):
    L, x, g, _ = _layer(name)
    assert synth.parse_header(L.record(0))["fmt"] == synth.FMT_VQ4P
    for t in (0, 1):
        out, idx, _ = O.moe_layer(L, x[t], fma=0)
        assert np.array_equal(idx, g[f"idx{t}_cpu"])
        assert np.array_equal(bits(out), bits(g[f"out{t}_cpu"]))
        out1, idx1, _ = O.moe_layer(L, x[t], fma=1)
        assert np.array_equal(idx1, g[f"idx{t}_avx512"])
        # the AVX-512 shared expert sums in another order
        assert rel_l2(out1, g[f"out{t}_avx512"]) < 1e-6


@pytest.mark.parametrize("name", list(VQ4P_MOE_CASES))
def test_vq4p_moe_chunk_golden(name):
    L, x, g, T = _layer(name)
    for tag, fma in (("cpu", 0), ("avx512", 1)):
        out, route, rw = O.moe_chunk(L, x[:T], fma=fma)
        assert np.array_equal(route, g[f"route_{tag}"])
        assert np.array_equal(bits(out), bits(g[f"chunk_{tag}"]))


@pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built here")
@pytest.mark.parametrize("seed", [1, 2, 3])
def test_vq4p_restatement_vs_reference_live(seed):
    rng = np.random.default_rng(seed)
    raw = synth.codebooks(rng, 8, entries=64)
    books = synth.flush_f16(raw)
    N = 8 * int(rng.integers(1, 200))
    M = int(rng.integers(1, 300))
    x = synth.activations(seed + 300, N)[0]
    idx, sc = synth.random_matrix(rng, M, N, stages=4)
    y = O.vq4p_matvec(idx, sc, x, M, N, books, 2, fma=1)
    yr = O.ref_vq4p_matvec(idx, sc, x, M, N, books, 2)
    assert np.array_equal(bits(y), bits(yr))
