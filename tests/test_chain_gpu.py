"""Layers chained on one stream, as a decode step runs them.

The decode step feeds each layer the residual stream the previous layer
left (src/model.c:3927-3945): norm = rmsnorm(h), h += moe_layer(norm). The
library's MoE block does that on the device (waste_cuda_moe_block_dev), so
the output buffer of one layer's call is the input of the next, on the same
stream, with nothing on the host between them. These tests hold such chains
to the oracle's own chain (oracle.moe_block, which restates the reference's
rmsnorm and moe_layer):
  * every layer's route bit-exact, and its MoE part (h_out - h) within 2e-5
    relative L2 of the oracle on the same input;
  * the device chain within 2e-5 of the oracle's chain from the same h0 at
    every layer;
  * the same chain launched directly and replayed from a CUDA graph (twice,
    with new inputs);
  * batches of 3 and 17 tokens (the decode-sized and the batched kernel
    forms) and the host-buffer block call.
"""
import numpy as np
import pytest

import oracle as O
from golden_cases import rel_l2
from warp_b200 import synth

pytestmark = pytest.mark.gpu
TOL = 2e-5
N_LAYERS = 8
FIRST = 61


@pytest.fixture(scope="module")
def chain(cuda_lib):
    wb = cuda_lib
    base = synth.moe_layer(601, hidden=1024, inter=512, n_experts=64, top_k=8, shared_inter=512,
                           layer=FIRST, with_bias=True)
    layers, norms = [], []
    wb.codebooks_load_f16(base.books_raw)
    for k in range(N_LAYERS):
        L = base if k == 0 else synth.derive_layer(base, FIRST + k, 610 + k)
        nw = synth.norm_weight(620 + k, L.hidden)
        wb.vq_bank_free(L.layer)
        wb.vq_bank_load(L.layer, L.n_experts, L.rec_bytes, 0, L.n_experts, L.bank, L.inter,
                        L.hidden, L.stages)
        wb.moe_trunk_load(L.layer, L.n_experts, L.hidden, L.top_k, L.renorm, L.routed_scale,
                          L.router, L.bias, L.shared_inter, L.sh)
        wb.moe_norm_load(L.layer, nw, synth.NORM_EPS)
        layers.append(L)
        norms.append(nw)
    yield wb, layers, norms
    for L in layers:
        wb.vq_bank_free(L.layer)


def _oracle_chain(layers, norms, h0):
    hs, idx = [np.asarray(h0, np.float32)], []
    for L, nw in zip(layers, norms):
        h, i, _ = O.moe_block(L, hs[-1], nw, synth.NORM_EPS)
        hs.append(h)
        idx.append(i)
    return hs, idx


def _check(layers, norms, hs_dev, idx_dev, h0):
    """Per layer against the oracle on the device's own input, and the whole
    chain against the oracle's chain."""
    hs_o, idx_o = _oracle_chain(layers, norms, h0)
    assert np.array_equal(hs_dev[0], np.asarray(h0, np.float32))
    for k, (L, nw) in enumerate(zip(layers, norms)):
        ro, ri, _ = O.moe_block(L, hs_dev[k], nw, synth.NORM_EPS)
        assert np.array_equal(idx_dev[k], ri), (k, idx_dev[k], ri)
        assert rel_l2(hs_dev[k + 1] - hs_dev[k], ro - hs_dev[k]) < TOL, k
        assert np.array_equal(idx_dev[k], idx_o[k]), k
        assert rel_l2(hs_dev[k + 1], hs_o[k + 1]) < TOL, k


def _launch_chain(wb, layers, hs, idx, w, stream):
    for k, L in enumerate(layers):
        wb.moe_block_dev(L.layer, 1, hs[k].data_ptr(), hs[k + 1].data_ptr(), idx[k].data_ptr(),
                         w[k].data_ptr(), stream)


def test_chain_direct_and_graph(chain):
    import torch
    wb, layers, norms = chain
    H = layers[0].hidden
    dev = torch.device("cuda", 0)
    hs = torch.zeros((N_LAYERS + 1, H), dtype=torch.float32, device=dev)
    idx = torch.zeros((N_LAYERS, layers[0].top_k), dtype=torch.int32, device=dev)
    w = torch.zeros((N_LAYERS, layers[0].top_k), dtype=torch.float32, device=dev)
    s = torch.cuda.Stream(device=dev)
    h0 = synth.activations(630, H)[0]
    hs[0].copy_(torch.from_numpy(h0))
    torch.cuda.synchronize()
    _launch_chain(wb, layers, hs, idx, w, s.cuda_stream)      # direct launches
    torch.cuda.synchronize()
    assert wb.device_errors() == 0
    _check(layers, norms, hs.cpu().numpy(), idx.cpu().numpy(), h0)

    g = torch.cuda.CUDAGraph()                                 # the same chain, captured
    with torch.cuda.graph(g, stream=s, capture_error_mode="thread_local"):
        _launch_chain(wb, layers, hs, idx, w, s.cuda_stream)
    for rep in range(2):
        h0 = synth.activations(631 + rep, H)[0]
        hs.zero_()
        hs[0].copy_(torch.from_numpy(h0))
        torch.cuda.synchronize()
        g.replay()
        torch.cuda.synchronize()
        assert wb.device_errors() == 0
        _check(layers, norms, hs.cpu().numpy(), idx.cpu().numpy(), h0)
    del g


@pytest.mark.parametrize("T", [3, 17])
def test_chain_batches(chain, T):
    """T tokens per call through three chained layers (17: the many-token
    router and the separate SiLU kernel), in place: d_h_out == d_h."""
    import torch
    wb, layers, norms = chain
    H, K = layers[0].hidden, layers[0].top_k
    dev = torch.device("cuda", 0)
    h0 = synth.activations(640 + T, H, T=T)
    h = torch.from_numpy(h0.copy()).to(dev)
    idx = torch.zeros((3, T, K), dtype=torch.int32, device=dev)
    w = torch.zeros((3, T, K), dtype=torch.float32, device=dev)
    snaps = [h0.copy()]
    for k in range(3):
        wb.moe_block_dev(layers[k].layer, T, h.data_ptr(), h.data_ptr(), idx[k].data_ptr(),
                         w[k].data_ptr())
        torch.cuda.synchronize()
        snaps.append(h.cpu().numpy())
    assert wb.device_errors() == 0
    ih = idx.cpu().numpy()
    for t in range(T):
        _check(layers[:3], norms[:3], [sn[t] for sn in snaps], [ih[k, t] for k in range(3)],
               h0[t])


def test_block_host_call(chain):
    """waste_cuda_moe_block: host buffers in and out, chained on the host."""
    wb, layers, norms = chain
    h0 = synth.activations(650, layers[0].hidden)[0]
    hs, ids = [h0], []
    for L in layers[:4]:
        h, i, _ = wb.moe_block(L.layer, hs[-1], L.top_k, L.hidden)
        hs.append(h)
        ids.append(i)
    _check(layers[:4], norms[:4], hs, ids, h0)
