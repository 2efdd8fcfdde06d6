"""The VQ3R matvec with interleaved table copies (waste_cuda_vq_matvec_sel_dev)
against the plain batched matvec and the oracle.

Each table entry is held 2 or 4 times and every lookup reads the copy a
per-matrix copy-select stream names (written once by
waste_cuda_vq_sel_build_dev). The table values and the summation order are
those of waste_cuda_vq_matvec_dev, so the results must be the same bits, and
within 2e-5 relative L2 of the oracle (src/model.c:1956-2024)."""
import numpy as np
import pytest

import oracle as O
from golden_cases import bits, rel_l2
from warp_b200 import synth

pytestmark = pytest.mark.gpu
TOL = 2e-5


@pytest.mark.parametrize("M,N", [(4096, 4096), (7168, 2048), (2304, 1024), (3000, 520)])
@pytest.mark.parametrize("copies", [2, 4])
def test_matvec_sel_bitexact(cuda_lib, M, N, copies):
    import torch
    wb = cuda_lib
    rng = np.random.default_rng(M + N + copies)
    raw = synth.codebooks(rng, 3)
    wb.codebooks_load_f16(raw)
    G = 3
    mats = [synth.random_matrix(rng, M, N) for _ in range(G)]
    xs = synth.activations(M + copies, N, T=G)
    dev = torch.device("cuda", 0)
    d_idx = [torch.from_numpy(m[0]).to(dev) for m in mats]
    d_sc = [torch.from_numpy(m[1].view(np.int16)).to(dev) for m in mats]
    d_x = torch.from_numpy(xs).to(dev)
    nb = wb.vq_sel_bytes(M, N, 3, copies)
    assert nb > 0
    d_sel = [torch.empty(nb, dtype=torch.uint8, device=dev) for _ in range(G)]
    for g in range(G):
        wb.vq_sel_build_dev(d_idx[g].data_ptr(), d_sel[g].data_ptr(), M, N, 3, copies)
    y0 = torch.empty((G, M), device=dev)
    y1 = torch.full((G, M), float("nan"), device=dev)
    ptrs = ([t.data_ptr() for t in d_idx], [t.data_ptr() for t in d_sc],
            [d_x[g].data_ptr() for g in range(G)])
    wb.vq_matvec_dev(*ptrs, [y0[g].data_ptr() for g in range(G)], M, N, 0, 3)
    wb.vq_matvec_sel_dev(ptrs[0], [t.data_ptr() for t in d_sel], ptrs[1], ptrs[2],
                         [y1[g].data_ptr() for g in range(G)], M, N, 0, 3, copies)
    torch.cuda.synchronize()
    a, b = y0.cpu().numpy(), y1.cpu().numpy()
    assert np.array_equal(bits(a), bits(b))
    for g in range(G):
        yo = O.vq_matvec(mats[g][0], mats[g][1], xs[g], M, N, synth.flush_f16(raw), 0)
        assert rel_l2(b[g], yo) < TOL


def test_matvec_sel_refuses_small(cuda_lib):
    wb = cuda_lib
    assert wb.vq_sel_bytes(1024, 2304, 3, 2) == 0      # one tile would not hold the rows
    assert wb.vq_sel_bytes(4096, 4096, 3, 3) == 0      # 2 or 4 copies only
