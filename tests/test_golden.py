"""The CPU restatement (oracle/) against the reference's golden vectors.

The fixtures in tests/golden/ were produced by the reference engine compiled
from its own sources (tests/golden/make_golden.py). The restatement must
reproduce them bit for bit wherever it follows the same backend's
arithmetic: the portable (WASTE_BACKEND=cpu) goldens with fma=0, the AVX-512
goldens with fma=1. The one place the AVX-512 engine sums in an order the
restatement does not follow is the shared expert's 16-lane Q8G dot product
(src/simd_avx512.c:20-88), so whole-layer AVX-512 outputs are held to 1e-6.
"""
import numpy as np
import pytest

import oracle as O
from golden_cases import MATVEC_CASES, MOE_CASES, bits, load, rel_l2
from warp_b200 import synth


def test_f16_flush_all_patterns():
    g = load("f16_flush")["bits"]
    allpat = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    assert np.array_equal(bits(O.f16_flush(allpat)), g)
    assert np.array_equal(bits(synth.flush_f16(allpat)), g)
    # subnormals flush to a signed zero, normals decode exactly
    sub = allpat[((allpat >> 10) & 0x1F) == 0]
    assert np.all(np.abs(synth.flush_f16(sub)) == 0)


@pytest.mark.parametrize("tag,fma", [("avx512", 1), ("cpu", 0)])
def test_lut_golden(tag, fma):
    g = load(f"lut_{tag}")
    books = synth.flush_f16(g["books_raw"])
    lut = O.lut_build(books, int(g["cb_base"]), g["x"], fma=fma)
    assert np.array_equal(bits(lut), bits(g["lut"]))


@pytest.mark.parametrize("case", MATVEC_CASES)
@pytest.mark.parametrize("tag,fma", [("avx512", 1), ("cpu", 0)])
def test_matvec_golden(case, tag, fma):
    g = load(f"{case}_{tag}")
    books = synth.flush_f16(g["books_raw"])
    y = O.vq_matvec(g["idx"], g["scale"], g["x"], int(g["M"]), int(g["N"]), books,
                    int(g["cb_base"]), int(g["stages"]), fma=fma)
    assert np.array_equal(bits(y), bits(g["y"]))


def _layer(name):
    from golden.make_golden import layer_sha
    seed, kw, xseed, T = MOE_CASES[name]
    L = synth.moe_layer(seed, **kw)
    g = load(name)
    assert layer_sha(L) == str(g["sha"]), "synthetic generator drifted from the fixture"
    x = synth.activations(xseed, L.hidden, T=max(T, 2))
    return L, x, g, T


@pytest.mark.parametrize("name", list(MOE_CASES))
def test_moe_layer_golden(name):
    L, x, g, _ = _layer(name)
    for t in (0, 1):
        out, idx, w = O.moe_layer(L, x[t], fma=0)
        assert np.array_equal(idx, g[f"idx{t}_cpu"])
        assert np.array_equal(bits(out), bits(g[f"out{t}_cpu"]))
        out1, idx1, _ = O.moe_layer(L, x[t], fma=1)
        assert np.array_equal(idx1, g[f"idx{t}_avx512"])
        assert rel_l2(out1, g[f"out{t}_avx512"]) < 1e-6


@pytest.mark.parametrize("name", [n for n, c in MOE_CASES.items() if c[3]])
def test_moe_chunk_golden(name):
    L, x, g, T = _layer(name)
    for tag, fma in (("cpu", 0), ("avx512", 1)):
        out, route, rw = O.moe_chunk(L, x[:T], fma=fma)
        assert np.array_equal(route, g[f"route_{tag}"])
        assert np.array_equal(bits(rw), bits(g[f"rw_{tag}"]))
        assert np.array_equal(bits(out), bits(g[f"chunk_{tag}"]))


def test_route_ties_and_nan():
    # strict >: the lowest index wins a tie; NaN is never selected
    lg = np.array([0.5, 2.0, 2.0, np.nan, 1.0], np.float32)
    idx, w = O.route(lg, None, 3, 0, 1.0)
    assert list(idx) == [1, 2, 4]
    idx, w = O.route(lg, np.array([0, 0, 0.5, 0, 0], np.float32), 2, 1, 2.0)
    assert list(idx) == [2, 1]
    assert abs(float(w.sum()) - 2.0) < 1e-6


@pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built here")
@pytest.mark.parametrize("seed", [1, 2, 3])
def test_restatement_vs_reference_live(seed):
    """Fresh seeds straight through the compiled reference."""
    R = O.ref()
    rng = np.random.default_rng(seed)
    raw = synth.codebooks(rng, 9)
    books = synth.flush_f16(raw)
    N = 8 * int(rng.integers(4, 40))
    M = int(rng.integers(1, 300))
    x = synth.activations(seed + 100, N)[0]
    idx, sc = synth.random_matrix(rng, M, N)
    for be, fma in ((R.refh_best_backend(), 1 if R.refh_best_backend() else 0), (0, 0)):
        R.refh_set_backend(be)
        y = np.empty(M, np.float32)
        R.refh_vq_matvec(O._p(y), O._p(idx), O._p(sc), O._p(x), M, N, O._p(books), 9, 3,
                         3, 256, 8)
        yo = O.vq_matvec(idx, sc, x, M, N, books, 3, fma=fma)
        assert np.array_equal(bits(y), bits(yo))


def test_rmsnorm_golden():
    """The MoE block's rmsnorm (src/model.c:132-138) bit for bit."""
    from golden_cases import NORM_SIZES
    g = load("norm")
    for n in NORM_SIZES:
        o = O.rmsnorm(g[f"x{n}"], g[f"w{n}"], float(g["eps"]))
        assert np.array_equal(bits(o), bits(g[f"out{n}"])), n


@pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built here")
def test_rmsnorm_vs_reference_live():
    x = synth.activations(5, 4096)[0] * np.float32(0.01)
    w = synth.norm_weight(6, 4096)
    assert np.array_equal(bits(O.rmsnorm(x, w, 1e-5)), bits(O.ref_rmsnorm(x, w, 1e-5)))


def test_situ_golden_is_situ():
    """The SiTU fixture really took the SiTU path: the SiLU restatement of
    the same layer disagrees with it, the SiTU restatement matches."""
    import copy
    L, x, g, _ = _layer("moe_situ")
    assert L.act_situ == 1
    L0 = copy.copy(L)
    L0.act_situ = 0
    o_silu, _, _ = O.moe_layer(L0, x[0], fma=0)
    o_situ, _, _ = O.moe_layer(L, x[0], fma=0)
    assert rel_l2(o_silu, g["out0_cpu"]) > 1e-3
    assert np.array_equal(bits(o_situ), bits(g["out0_cpu"]))


@pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built here")
def test_situ_pair_vs_reference_live():
    rng = np.random.default_rng(3)
    g = (rng.standard_normal(2000) * 6).astype(np.float32)
    u = (rng.standard_normal(2000) * 40).astype(np.float32)
    for beta, lbeta in ((4.0, 25.0), (1.0, 0.0), (2.5, -1.0)):
        assert np.array_equal(bits(O.situ_pair(g, u, beta, lbeta)),
                              bits(O.ref_situ_pair(g, u, beta, lbeta)))


def test_mvq_golden():
    """The trunk matvec (src/model.c:265-320, Q8G/Q4G/Q3G) bit for bit."""
    from golden_cases import MVQ_CASES
    g = load("mvq")
    for name, (rows, inp, nb) in MVQ_CASES.items():
        y = O.mvq_rows(g[f"{name}_raw"], g[f"{name}_s"], g[f"{name}_x"], inp, 128, nb,
                       int(g[f"{name}_rowbytes"]))
        assert np.array_equal(bits(y), bits(g[f"{name}_y"])), name


@pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built here")
def test_mvq_vs_reference_live():
    rng = np.random.default_rng(11)
    for nb in (8, 4, 3):
        raw, s, rb = synth.trunk_tensor(rng, 40, 777, nb)
        x = synth.activations(12 + nb, 777)[0]
        assert np.array_equal(bits(O.mvq_rows(raw, s, x, 777, 128, nb, rb)),
                              bits(O.ref_mvq_rows(raw, s, x, 777, 128, nb, rb)))
