"""The converter's RVQ encoder on the device (warp_b200/csrc/vq_encode.cu)
against the reference's own outputs (tests/golden/enc.npz): codes and
Lloyd centroids bit for bit (the distances are summed in the CPU's order
with IEEE operations, and the centroid sums keep the vector order through
a stable sort by cluster)."""
import numpy as np
import pytest

import oracle as O
from golden_cases import ENC_CASES, LLOYD_CASES, bits, enc_inputs, load, lloyd_inputs

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", list(ENC_CASES))
def test_encode_bitexact(cuda_lib, name):
    g = load("enc")
    X, books = enc_inputs(name)
    assert np.array_equal(cuda_lib.vq_encode(X, books), g[f"{name}_codes"])


@pytest.mark.parametrize("name", list(LLOYD_CASES))
def test_lloyd_bitexact(cuda_lib, name):
    g = load("enc")
    X, C0 = lloyd_inputs(name)
    C, live = cuda_lib.vq_lloyd(X, C0)
    assert live == int(g[f"{name}_live"])
    assert np.array_equal(bits(C), bits(g[f"{name}_C"]))


def test_encode_expert_matrix_dev(cuda_lib):
    """A whole Kimi-Linear gate matrix's vectors (1024 x 2304 / 8) through
    three stages on device pointers, against the restatement."""
    import torch
    wb = cuda_lib
    rng = np.random.default_rng(5)
    X = np.clip(rng.normal(0.0, 0.4, (1024 * 2304 // 8, 8)), -1, 1).astype(np.float32)
    books = np.stack([rng.normal(0.0, 0.3 / (s + 1), (256, 8)) for s in range(3)]
                     ).astype(np.float32)
    dev = torch.device("cuda", 0)
    dX, dB = torch.from_numpy(X).to(dev), torch.from_numpy(books).to(dev)
    dO = torch.empty((X.shape[0], 3), dtype=torch.uint8, device=dev)
    wb.vq_encode_dev(dX.data_ptr(), X.shape[0], dB.data_ptr(), 3, 256, 8, dO.data_ptr(),
                     torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert np.array_equal(dO.cpu().numpy(), O.vq_encode(X, books))


def test_encode_refuses_out_of_range(cuda_lib):
    wb = cuda_lib
    X = np.zeros((4, 8), np.float32)
    with pytest.raises(wb.WasteCudaError) as e:
        wb.vq_encode(X, np.zeros((1, 300, 8), np.float32))       # more than 256 entries
    assert e.value.rc == wb.E_ARG
