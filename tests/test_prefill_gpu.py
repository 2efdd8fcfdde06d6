"""The prefill expert loop on the tensor cores (tcgen05), against the oracle.

Routes are drawn from Zipf(1.1) over a seeded permutation of the experts, so
a few experts get many tokens and many get one or none — the skew of BASELINE
config 3. Per token the oracle adds the experts in ascending id, as
moe_chunk does (src/model.c:3632-3656); the device result must be within
2e-5 relative L2 (it computes with split-fp16 tensor-core contractions).
"""
import numpy as np
import pytest

import oracle as O
from golden_cases import rel_l2
from warp_b200 import synth

pytestmark = pytest.mark.gpu
TOL = 2e-5


def _ascending(L, idx, w, x):
    o = np.argsort(idx, kind="stable")
    return O.moe_experts(L, idx[o].astype(np.int32), w[o].astype(np.float32), x, fma=1)


@pytest.mark.parametrize("T,act", [(128, 0), (40, 0), (512, 0), (128, 1)])
def test_prefill_tc_kimi_shape_zipf(cuda_lib, T, act):
    """T = 512 is config 3's size; act 1 is K3's SiTU in the gate/up -> down
    hand-off."""
    import torch
    wb = cuda_lib
    # hidden 2304, inter 1024, 256 experts, top-8
    L = synth.moe_layer(1234, act_situ=act)
    wb.vq_bank_free(L.layer)
    wb.load_layer(L, trunk=False)
    route = synth.zipf_routes(77 + T, T, L.n_experts, L.top_k).astype(np.int32)
    rng = np.random.default_rng(78 + T)
    rw = rng.uniform(0.05, 0.6, size=route.shape).astype(np.float32)
    x = synth.activations(79 + T, L.hidden, T=T)
    dev = torch.device("cuda", 0)
    d_r, d_w = torch.from_numpy(route).to(dev), torch.from_numpy(rw).to(dev)
    d_x = torch.from_numpy(x).to(dev)
    d_o = torch.full((T, L.hidden), float("nan"), device=dev)
    wb.moe_prefill_dev(L.layer, T, L.top_k, d_r.data_ptr(), d_w.data_ptr(), d_x.data_ptr(),
                       d_o.data_ptr())
    torch.cuda.synchronize()
    assert wb.device_errors() == 0
    out = d_o.cpu().numpy()
    worst = 0.0
    for t in range(T):
        ref = _ascending(L, route[t], rw[t], x[t])
        worst = max(worst, rel_l2(out[t], ref))
    assert worst < TOL, worst
    # the host slot (the tensor cores for a full chunk, lookups below two
    # tokens per expert) agrees within the same tolerance
    y = wb.moe_chunk_experts(L.layer, route[:64], rw[:64], x[:64], L.hidden, L.inter, act,
                             L.situ_beta, L.situ_lbeta)
    assert max(rel_l2(y[t], out[t]) for t in range(min(T, 64))) < TOL
    wb.vq_bank_free(L.layer)


def test_prefill_tc_refuses_unsupported(cuda_lib):
    """Rows not a multiple of 128 stay on the lookup path: the device entry
    point refuses them instead of computing something else."""
    import torch
    wb = cuda_lib
    L = synth.moe_layer(11, hidden=192, inter=96, n_experts=12, top_k=3, shared_inter=0, layer=13)
    wb.vq_bank_free(L.layer)
    wb.load_layer(L, trunk=False)
    T = 8
    r = torch.zeros((T, 3), dtype=torch.int32, device="cuda")
    w = torch.zeros((T, 3), device="cuda")
    x = torch.zeros((T, 192), device="cuda")
    o = torch.zeros((T, 192), device="cuda")
    with pytest.raises(wb.WasteCudaError) as e:
        wb.moe_prefill_dev(L.layer, T, 3, r.data_ptr(), w.data_ptr(), x.data_ptr(), o.data_ptr())
    assert e.value.rc == wb.E_ARG
    wb.vq_bank_free(L.layer)
