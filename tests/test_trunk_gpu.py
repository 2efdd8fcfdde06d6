"""The trunk matvec on the device (the engine's mvq_rows_f32 slot,
src/model.c:265-320), against the reference's own compiled kernel.

waste_cuda_mvq_rows_dev on Q8G, Q4G and Q3G tensors — the goldens written by
the reference's waste_mvq_rows_f32 (tests/golden/mvq.npz, regular and ragged
widths) and a large Kimi-Linear lm_head slice — within 2e-5 relative L2
(fp32, another summation order), and a row range [r0, r1) writes only those
rows."""
import numpy as np
import pytest

import oracle as O
from golden_cases import load, rel_l2
from warp_b200 import synth

pytestmark = pytest.mark.gpu
TOL = 2e-5


def _run(wb, raw, s, x, inp, bits, rb, r0=0, r1=None):
    import torch
    dev = torch.device("cuda", 0)
    rows = raw.shape[0]
    r1 = rows if r1 is None else r1
    dW = torch.from_numpy(np.ascontiguousarray(raw)).to(dev)
    ds = torch.from_numpy(np.ascontiguousarray(s).view(np.int16)).to(dev)
    dx = torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    dy = torch.full((rows,), float("nan"), device=dev)
    wb.mvq_rows_dev(dy.data_ptr(), dW.data_ptr(), ds.data_ptr(), dx.data_ptr(), r0, r1, inp, 128,
                    bits, rb)
    torch.cuda.synchronize()
    return dy.cpu().numpy()


def test_mvq_golden_on_device(cuda_lib):
    from golden_cases import MVQ_CASES
    wb = cuda_lib
    g = load("mvq")
    for name, (rows, inp, nb) in MVQ_CASES.items():
        y = _run(wb, g[f"{name}_raw"], g[f"{name}_s"], g[f"{name}_x"], inp, nb,
                 int(g[f"{name}_rowbytes"]))
        assert rel_l2(y, g[f"{name}_y"]) < TOL, name


@pytest.mark.parametrize("bits", [8, 4])
def test_mvq_lm_head_slice(cuda_lib, bits):
    """8192 rows at the lm_head width (hidden 2304), and a row range."""
    wb = cuda_lib
    rng = np.random.default_rng(100 + bits)
    raw, s, rb = synth.trunk_tensor(rng, 8192, 2304, bits)
    x = synth.activations(101, 2304)[0]
    yo = O.mvq_rows(raw, s, x, 2304, 128, bits, rb)
    y = _run(wb, raw, s, x, 2304, bits, rb)
    assert rel_l2(y, yo) < TOL
    part = _run(wb, raw, s, x, 2304, bits, rb, 1000, 3000)
    assert np.isnan(part[:1000]).all() and np.isnan(part[3000:]).all()
    assert rel_l2(part[1000:3000], yo[1000:3000]) < TOL
