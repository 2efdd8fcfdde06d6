"""Parity of the CUDA backend (through the C ABI) against the oracle.

Tolerances, as the north star states them:
  * the codebook table (LUT), the dequantised weights and the routing
    indices are bit-exact;
  * matvec and layer outputs are within 2e-5 relative L2 (fp32 accumulation,
    different summation order over vector positions).
The oracle is the CPU restatement pinned to the reference's golden vectors
(tests/test_golden.py); the goldens themselves are checked here too.
"""
import numpy as np
import pytest

import oracle as O
from golden_cases import MATVEC_CASES, MOE_CASES, bits, load, rel_l2
from warp_b200 import synth

pytestmark = pytest.mark.gpu
TOL = 2e-5


def test_backend_registers(cuda_lib):
    wb = cuda_lib
    name = wb.register_cuda()
    assert name and "sm_100a" in name
    slots = wb.register_cuda_vq()
    assert slots.moe_experts and slots.moe_chunk_experts and slots.vq_bank_load


@pytest.mark.parametrize("tag", ["avx512"])
def test_lut_bitexact(cuda_lib, tag):
    wb = cuda_lib
    g = load(f"lut_{tag}")
    wb.codebooks_load_f16(g["books_raw"])
    lut = wb.lutb(g["x"], int(g["cb_base"]))
    assert np.array_equal(bits(lut), bits(g["lut"]))
    # and at a larger, freshly seeded size
    rng = np.random.default_rng(77)
    raw = synth.codebooks(rng, 6)
    wb.codebooks_load_f16(raw)
    x = synth.activations(78, 4096)[0]
    assert np.array_equal(bits(wb.lutb(x, 3)), bits(O.lut_build(synth.flush_f16(raw), 3, x)))


@pytest.mark.parametrize("M,N,st", [(100, 256, 3), (256, 512, 3), (64, 8, 3), (130, 96, 2),
                                    (4096, 4096, 3)])
def test_dequant_bitexact(cuda_lib, M, N, st):
    wb = cuda_lib
    rng = np.random.default_rng(M * 7 + N)
    raw = synth.codebooks(rng, 9)
    wb.codebooks_load_f16(raw)
    idx, sc = synth.random_matrix(rng, M, N, stages=st)
    W = wb.vq_dequant(idx, sc, M, N, 3, st)
    Wo = O.dequant(idx, sc, M, N, synth.flush_f16(raw), 3, st)
    assert np.array_equal(bits(W), bits(Wo))


@pytest.mark.parametrize("case", MATVEC_CASES)
def test_matvec_golden(cuda_lib, case):
    wb = cuda_lib
    g = load(f"{case}_avx512")
    wb.codebooks_load_f16(g["books_raw"])
    y = wb.vq_matvec(g["idx"], g["scale"], g["x"], int(g["M"]), int(g["N"]), int(g["cb_base"]),
                     int(g["stages"]))
    assert rel_l2(y, g["y"]) < TOL


@pytest.mark.parametrize("M,N", [(4096, 4096), (1024, 2304), (2304, 1024), (7168, 2048),
                                 (64, 8), (1, 64)])
def test_matvec_shapes(cuda_lib, M, N):
    """Config 1 (4096x4096) and the Kimi-Linear / K3-class expert shapes."""
    wb = cuda_lib
    rng = np.random.default_rng(M + N)
    raw = synth.codebooks(rng, 3)
    wb.codebooks_load_f16(raw)
    idx, sc = synth.random_matrix(rng, M, N)
    x = synth.activations(5, N)[0]
    y = wb.vq_matvec(idx, sc, x, M, N, 0)
    yo = O.vq_matvec(idx, sc, x, M, N, synth.flush_f16(raw), 0)
    assert rel_l2(y, yo) < TOL
    # deterministic: the same call twice gives the same bits
    assert np.array_equal(bits(wb.vq_matvec(idx, sc, x, M, N, 0)), bits(y))


def test_matvec_dev_batched(cuda_lib):
    """The device-pointer batched entry point over G independent matrices."""
    import torch
    wb = cuda_lib
    M, N, G = 1024, 2304, 5
    rng = np.random.default_rng(9)
    raw = synth.codebooks(rng, 3)
    wb.codebooks_load_f16(raw)
    mats = [synth.random_matrix(rng, M, N) for _ in range(G)]
    xs = synth.activations(10, N, T=G)
    d_idx = [torch.from_numpy(m[0]).cuda() for m in mats]
    d_sc = [torch.from_numpy(m[1].view(np.int16)).cuda() for m in mats]
    d_x = torch.from_numpy(xs).cuda()
    d_y = torch.empty((G, M), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    wb.vq_matvec_dev([t.data_ptr() for t in d_idx], [t.data_ptr() for t in d_sc],
                     [d_x[g].data_ptr() for g in range(G)], [d_y[g].data_ptr() for g in range(G)],
                     M, N, 0, 3, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    y = d_y.cpu().numpy()
    for g in range(G):
        yo = O.vq_matvec(mats[g][0], mats[g][1], xs[g], M, N, synth.flush_f16(raw), 0)
        assert rel_l2(y[g], yo) < TOL


def _layer(name):
    seed, kw, xseed, T = MOE_CASES[name]
    L = synth.moe_layer(seed, **kw)
    x = synth.activations(xseed, L.hidden, T=max(T, 2))
    return L, x, load(name), T


@pytest.mark.parametrize("name", list(MOE_CASES))
def test_moe_layer_parity(cuda_lib, name):
    """Router + routed experts + shared expert on the device: expert indices
    bit-exact against the reference's golden route, output within 2e-5 of
    the reference's (AVX-512) output."""
    wb = cuda_lib
    L, x, g, _ = _layer(name)
    wb.vq_bank_free(L.layer)
    wb.load_layer(L)
    for t in (0, 1):
        out, idx, w = wb.moe_layer(L.layer, x[t], L.top_k, L.hidden)
        assert np.array_equal(idx, g[f"idx{t}_avx512"])
        assert rel_l2(out, g[f"out{t}_avx512"]) < TOL
        _, _, wo = O.moe_layer(L, x[t], fma=1)
        assert rel_l2(w, wo) < 1e-6


@pytest.mark.parametrize("name", list(MOE_CASES))
def test_moe_experts_parity(cuda_lib, name):
    """The drop-in slot: route given by the engine, host buffers in and out."""
    wb = cuda_lib
    L, x, g, _ = _layer(name)
    wb.vq_bank_free(L.layer)
    wb.load_layer(L, trunk=False)
    _, idx, w = O.moe_layer(L, x[0], fma=1)
    y = wb.moe_experts(L.layer, idx, w, x[0], L.hidden, L.inter, L.act_situ, L.situ_beta,
                       L.situ_lbeta)
    yo = O.moe_experts(L, idx, w, x[0], fma=1)
    assert rel_l2(y, yo) < TOL


@pytest.mark.parametrize("name", [n for n, c in MOE_CASES.items() if c[3]])
def test_moe_chunk_parity(cuda_lib, name):
    """Prefill slot: per token, experts added in ascending id (moe_chunk)."""
    import copy
    wb = cuda_lib
    L, x, g, T = _layer(name)
    wb.vq_bank_free(L.layer)
    wb.load_layer(L, trunk=False)
    route, rw = g["route_avx512"], g["rw_avx512"]
    y = wb.moe_chunk_experts(L.layer, route, rw, x[:T], L.hidden, L.inter, L.act_situ,
                             L.situ_beta, L.situ_lbeta)
    L0 = copy.copy(L)
    L0.shared_inter = 0          # the routed part alone
    yo, r2, _ = O.moe_chunk(L0, x[:T], fma=1)
    assert np.array_equal(r2, route)
    assert rel_l2(y, yo) < TOL


def test_bank_rejects_bad_record(cuda_lib):
    wb = cuda_lib
    L = synth.moe_layer(21, hidden=128, inter=64, n_experts=4, top_k=2, shared_inter=0, layer=7)
    wb.vq_bank_free(7)
    wb.codebooks_load_f16(L.books_raw)
    bad = L.bank.copy()
    bad[L.rec_bytes + 4] ^= 0xFF           # expert 1's layer field
    with pytest.raises(wb.WasteCudaError) as e:
        wb.vq_bank_load(7, 4, L.rec_bytes, 0, 4, bad, 64, 128, 3)
    assert e.value.rc == wb.E_RECORD
    wb.vq_bank_load(7, 4, L.rec_bytes, 0, 4, L.bank, 64, 128, 3)
    with pytest.raises(wb.WasteCudaError) as e:
        wb.moe_experts(7, [0, 9], [1.0, 1.0], np.zeros(128, np.float32), 128, 64)
    assert e.value.rc == wb.E_ARG
    with pytest.raises(wb.WasteCudaError) as e:
        wb.moe_experts(8, [0, 1], [1.0, 1.0], np.zeros(128, np.float32), 128, 64)
    assert e.value.rc == wb.E_NOBANK
    wb.vq_bank_free(7)


def test_sharded_bank(cuda_lib):
    """A rank that owns half the experts loads only their records: routes
    over them match the oracle, a route naming an absent record is refused,
    and the whole-layer path (which may route anywhere) refuses the layer."""
    wb = cuda_lib
    L = synth.moe_layer(31, hidden=256, inter=128, n_experts=16, top_k=4, shared_inter=128,
                        layer=9)
    x = synth.activations(32, L.hidden)[0]
    wb.vq_bank_free(L.layer)
    wb.codebooks_load_f16(L.books_raw)
    half = L.n_experts // 2
    wb.vq_bank_load(L.layer, L.n_experts, L.rec_bytes, half, half,
                    L.bank[half * L.rec_bytes:], L.inter, L.hidden, L.stages)
    wb.moe_trunk_load(L.layer, L.n_experts, L.hidden, L.top_k, L.renorm, L.routed_scale,
                      L.router, L.bias, L.shared_inter, L.sh)
    idx = np.array([9, 15, 8, 12], np.int32)
    w = np.array([0.4, 0.3, 0.2, 0.1], np.float32)
    y = wb.moe_experts(L.layer, idx, w, x, L.hidden, L.inter)
    assert rel_l2(y, O.moe_experts(L, idx, w, x, fma=1)) < TOL
    with pytest.raises(wb.WasteCudaError) as e:
        wb.moe_experts(L.layer, [9, 3], [0.5, 0.5], x, L.hidden, L.inter)
    assert e.value.rc == wb.E_ARG
    with pytest.raises(wb.WasteCudaError) as e:
        wb.moe_layer(L.layer, x, L.top_k, L.hidden)
    assert e.value.rc == wb.E_ARG
    wb.vq_bank_load(L.layer, L.n_experts, L.rec_bytes, 0, half, L.bank, L.inter, L.hidden,
                    L.stages)
    out, ridx, _ = wb.moe_layer(L.layer, x, L.top_k, L.hidden)
    ro, rio, _ = O.moe_layer(L, x, fma=1)
    assert np.array_equal(ridx, rio) and rel_l2(out, ro) < TOL
    wb.vq_bank_free(L.layer)


@pytest.mark.parametrize("act", [0, 1])
def test_moe_layer_k3_shape(cuda_lib, act):
    """K3-class widths (hidden 7168, expert inter 2048, shared inter 2048,
    top-16) through the whole device layer and the prefill slot: the route
    bit-exact, outputs within 2e-5 of the oracle. 64 experts keep the bank
    near 1 GB; the 512-expert router is covered below. act 1: K3's own
    activation, SiTU (beta 4, linear beta 25), in the routed and shared
    experts."""
    wb = cuda_lib
    L = synth.moe_layer(77, hidden=7168, inter=2048, n_experts=64, top_k=16,
                        shared_inter=2048, layer=11, routed_scale=2.827, act_situ=act)
    x = synth.activations(78, L.hidden, T=3)
    wb.vq_bank_free(L.layer)
    wb.load_layer(L)
    out, idx, w = wb.moe_layer(L.layer, x[0], L.top_k, L.hidden)
    ro, ri, rw = O.moe_layer(L, x[0], fma=1)
    assert np.array_equal(idx, ri)
    assert rel_l2(out, ro) < TOL and rel_l2(w, rw) < 1e-6
    import copy
    L0 = copy.copy(L)
    L0.shared_inter = 0
    yo, route, rws = O.moe_chunk(L0, x, fma=1)
    y = wb.moe_chunk_experts(L.layer, route, rws, x, L.hidden, L.inter, act, L.situ_beta,
                             L.situ_lbeta)
    assert rel_l2(y, yo) < TOL
    # 17 tokens in one device call, the batched forms at this width: the
    # many-token router (x of four tokens per block at hidden 7168: groups
    # 4, 4, 4, 4, 1), 8-position gate/up slices, the separate SiLU kernel
    _batched_layer_check(wb, L, synth.activations(79, L.hidden, T=17))
    wb.vq_bank_free(L.layer)


def _batched_layer_check(wb, L, x):
    """T tokens through moe_layer_part_dev on a whole bank (shared expert
    for all of them): each token's route bit-exact, output within TOL."""
    import torch
    T = x.shape[0]
    dev = torch.device("cuda", 0)
    dx = torch.from_numpy(x).to(dev)
    o = torch.empty((T, L.hidden), device=dev)
    i = torch.empty((T, L.top_k), dtype=torch.int32, device=dev)
    w = torch.empty((T, L.top_k), device=dev)
    wb.moe_layer_part_dev(L.layer, T, dx.data_ptr(), o.data_ptr(), 0, T, i.data_ptr(),
                          w.data_ptr())
    torch.cuda.synchronize()
    assert wb.device_errors() == 0
    o, i = o.cpu().numpy(), i.cpu().numpy()
    for t in range(T):
        ro, ri, _ = O.moe_layer(L, x[t], fma=1)
        assert np.array_equal(i[t], ri), t
        assert rel_l2(o[t], ro) < TOL, t


def test_moe_layer_512_experts_top16(cuda_lib):
    """The router at 512 experts and top-16 (the K3 routing shape) on small
    experts: indices bit-exact, output within 2e-5."""
    wb = cuda_lib
    L = synth.moe_layer(91, hidden=256, inter=128, n_experts=512, top_k=16, shared_inter=128,
                        layer=12, with_bias=True)
    x = synth.activations(92, L.hidden, T=2)
    wb.vq_bank_free(L.layer)
    wb.load_layer(L)
    for t in range(2):
        out, idx, _ = wb.moe_layer(L.layer, x[t], L.top_k, L.hidden)
        ro, ri, _ = O.moe_layer(L, x[t], fma=1)
        assert np.array_equal(idx, ri)
        assert rel_l2(out, ro) < TOL
    # 17 tokens in one call: router token groups of eight, eight and one,
    # the separate SiLU kernel; 9 tokens: the decode-sized forms
    _batched_layer_check(wb, L, synth.activations(93, L.hidden, T=17))
    _batched_layer_check(wb, L, synth.activations(94, L.hidden, T=9))
    wb.vq_bank_free(L.layer)
