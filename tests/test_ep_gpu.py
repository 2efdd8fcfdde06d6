"""Expert parallelism on the device, through the C ABI, against the oracle.

  * one GPU, two banks holding the two halves of a layer's experts: the two
    partial outputs (the shared expert added by one of them) add up to the
    layer, and both see the same route;
  * one GPU, the NCCL path with a single rank (communicator of one);
  * two GPUs (skipped with fewer): tests/ep_worker.py under torchrun, each
    rank holding half the experts and checking its own tokens.
"""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

import oracle as O
from golden_cases import rel_l2
from warp_b200 import synth

pytestmark = pytest.mark.gpu
TOL = 2e-5
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_two_banks_partials_sum_to_layer(cuda_lib):
    import torch
    wb = cuda_lib
    L = synth.moe_layer(51, hidden=512, inter=256, n_experts=32, top_k=6, shared_inter=256,
                        layer=40, with_bias=True)
    D = synth.derive_layer(L, 41, 52)          # the same records under layer 41's headers
    T, E, h = 4, L.n_experts, L.n_experts // 2
    x = synth.activations(53, L.hidden, T=T)
    wb.codebooks_load_f16(L.books_raw)
    for lay, bank, first in ((40, L.bank, 0), (41, D.bank, h)):
        wb.vq_bank_free(lay)
        wb.vq_bank_reserve(lay, E, L.rec_bytes, first, h, L.inter, L.hidden, L.stages)
        wb.vq_bank_load(lay, E, L.rec_bytes, first, h, bank[first * L.rec_bytes:], L.inter,
                        L.hidden, L.stages)
        wb.moe_trunk_load(lay, E, L.hidden, L.top_k, L.renorm, L.routed_scale, L.router,
                          L.bias, L.shared_inter, L.sh)
    dev = torch.device("cuda", 0)
    dx = torch.from_numpy(x).to(dev)
    outs, idxs = [], []
    for lay, sh in ((40, (0, T)), (41, (0, 0))):
        o = torch.empty((T, L.hidden), device=dev)
        i = torch.empty((T, L.top_k), dtype=torch.int32, device=dev)
        w = torch.empty((T, L.top_k), device=dev)
        wb.moe_layer_part_dev(lay, T, dx.data_ptr(), o.data_ptr(), sh[0], sh[1], i.data_ptr(),
                              w.data_ptr())
        torch.cuda.synchronize()
        outs.append(o.cpu().numpy())
        idxs.append(i.cpu().numpy())
    assert wb.device_errors() == 0
    assert np.array_equal(idxs[0], idxs[1])
    for t in range(T):
        ro, ri, _ = O.moe_layer(L, x[t], fma=1)
        assert np.array_equal(idxs[0][t], ri)
        assert rel_l2(outs[0][t] + outs[1][t], ro) < TOL
    # a bank that holds only part of the layer is refused by the whole-layer path
    with pytest.raises(wb.WasteCudaError):
        wb.moe_layer(40, x[0], L.top_k, L.hidden)
    wb.vq_bank_free(40)
    wb.vq_bank_free(41)


def test_nccl_path_single_rank(cuda_lib):
    import torch
    wb = cuda_lib
    from warp_b200 import ep
    L = synth.moe_layer(61, hidden=512, inter=256, n_experts=32, top_k=6, shared_inter=256,
                        layer=42)
    T = 3
    x = synth.activations(62, L.hidden, T=T)
    ep.init(0, 1, ep.unique_id())
    try:
        wb.vq_bank_free(L.layer)
        wb.load_layer(L)
        dev = torch.device("cuda", 0)
        dx = torch.from_numpy(x).to(dev)
        out = torch.empty((T, L.hidden), device=dev)
        idx = torch.empty((T, L.top_k), dtype=torch.int32, device=dev)
        ep.moe_layer_dev(L.layer, T, dx.data_ptr(), out.data_ptr(), idx.data_ptr())
        torch.cuda.synchronize()
        out, idx = out.cpu().numpy(), idx.cpu().numpy()
        for t in range(T):
            ro, ri, _ = O.moe_layer(L, x[t], fma=1)
            assert np.array_equal(idx[t], ri)
            assert rel_l2(out[t], ro) < TOL
    finally:
        ep.shutdown()
        wb.vq_bank_free(L.layer)


def _gpus():
    import torch
    return torch.cuda.device_count()


@pytest.mark.skipif("_gpus() < 2")
def test_two_ranks_over_nccl():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node=2", "--master-addr", "127.0.0.1",
           "--master-port", str(port), os.path.join(ROOT, "tests", "ep_worker.py")]
    # the worker includes a rank that skips a call: no NVLink multicast in
    # any library while a rank may be out of step
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count("ep_worker ok") == 2, r.stdout[-2000:]
