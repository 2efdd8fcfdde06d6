"""The allocation-free batched matvec, waste_cuda_vq_matvec_dev_noalloc.

Some callers cannot allocate device memory once they are running. One kind
has reserved the device's memory for weights and state at load time, so a
late cudaMalloc can fail. Another cannot take the device-wide
synchronisation of cudaFree while other streams work. For them the
library offers a form of vq_matvec_dev that keeps its partial sums in a
fixed 32 MiB array built into the library instead of in growable scratch.

These tests call it through the C ABI and hold it to the existing entry
point on the same inputs. The checks:
  * two calls in a row agree with vq_matvec_dev within the matvec tolerance
    (2e-5 relative L2). The first call fills the array exactly
    (32 matrices of 4096 x 4096); the second has another shape, so its
    reads cannot lean on what the first left behind;
  * neither call takes device memory;
  * a call one matrix past the limit is refused with WASTE_CUDA_E_ARG before
    anything is launched;
  * in a fresh process, the FIRST call after init takes no device memory
    either: init has already brought the array and the kernels onto the
    device.
The module is named to run last, and it also passes on its own in a fresh
process.
"""
import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest

from golden_cases import rel_l2
from warp_b200 import synth

pytestmark = pytest.mark.gpu
TOL = 2e-5


def _case(torch, rng, G, M, N, n_distinct, xseed):
    """G matrix slots over n_distinct random matrices, a distinct x and y per
    slot, all on the device. Returns the pointer lists and the y tensors."""
    mats = [synth.random_matrix(rng, M, N) for _ in range(n_distinct)]
    d_idx = [torch.from_numpy(m[0]).cuda() for m in mats]
    d_sc = [torch.from_numpy(m[1].view(np.int16)).cuda() for m in mats]
    d_x = torch.from_numpy(synth.activations(xseed, N, T=G)).cuda()
    ptrs = ([d_idx[g % n_distinct].data_ptr() for g in range(G)],
            [d_sc[g % n_distinct].data_ptr() for g in range(G)],
            [d_x[g].data_ptr() for g in range(G)])
    return ptrs, (d_idx, d_sc, d_x)


def test_noalloc_matches_matvec_dev_two_calls(cuda_lib):
    import torch
    wb = cuda_lib
    rng = np.random.default_rng(2024)
    wb.codebooks_load_f16(synth.codebooks(rng, 3))
    stream = torch.cuda.current_stream().cuda_stream

    # call 1 fills the fixed array exactly; call 2 has another shape
    cases = [(32, 4096, 4096, 4, 31), (5, 1024, 2304, 5, 32)]
    built = []
    for G, M, N, nd, xseed in cases:
        assert G * -(-N // 64) * M * 4 <= wb.NOALLOC_SCRATCH_BYTES
        ptrs, keep = _case(torch, rng, G, M, N, nd, xseed)
        y_ref = torch.empty((G, M), dtype=torch.float32, device="cuda")
        y_new = torch.full((G, M), float("nan"), dtype=torch.float32, device="cuda")
        wb.vq_matvec_dev(*ptrs, [y_ref[g].data_ptr() for g in range(G)], M, N, 0, 3, stream)
        built.append((G, M, N, ptrs, keep, y_ref, y_new))
    torch.cuda.synchronize()

    for k, (G, M, N, ptrs, _, y_ref, y_new) in enumerate(built):
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        n0 = wb.launch_count()
        wb.vq_matvec_dev_noalloc(*ptrs, [y_new[g].data_ptr() for g in range(G)], M, N, 0, 3,
                                 stream)
        torch.cuda.synchronize()
        free1 = torch.cuda.mem_get_info()[0]
        assert wb.launch_count() - n0 == 2          # the library's own kernels ran
        assert free0 - free1 < (2 << 20), "the call took device memory"
        a, b = y_new.cpu().numpy(), y_ref.cpu().numpy()
        assert np.isfinite(a).all()
        for g in range(G):
            assert rel_l2(a[g], b[g]) < TOL, (k, g)


def test_noalloc_refuses_past_the_limit(cuda_lib):
    import torch
    wb = cuda_lib
    rng = np.random.default_rng(2025)
    wb.codebooks_load_f16(synth.codebooks(rng, 3))
    # 33 slots of 4096 x 4096: one matrix more than the array holds. Every
    # pointer is a real buffer of the right size, so the refusal is the only
    # thing that stands between this call and a launch.
    G, M, N = 33, 4096, 4096
    ptrs, keep = _case(torch, rng, G, M, N, 1, 33)
    y = torch.empty((M,), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    n0 = wb.launch_count()
    with pytest.raises(wb.WasteCudaError) as ei:
        wb.vq_matvec_dev_noalloc(*ptrs, [y.data_ptr()] * G, M, N, 0, 3,
                                 torch.cuda.current_stream().cuda_stream)
    assert ei.value.rc == wb.E_ARG
    assert "fixed" in str(ei.value)
    assert wb.launch_count() == n0


def test_noalloc_first_call_after_init_fresh_process():
    """A new process: device buffers first, then init, then free memory
    around the very first call of the entry point."""
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    code = textwrap.dedent("""
        import sys
        sys.path.insert(0, %r)
        import numpy as np, torch
        import warp_b200 as wb
        from warp_b200 import synth
        rng = np.random.default_rng(7)
        G, M, N = 4, 1024, 2304
        mats = [synth.random_matrix(rng, M, N) for _ in range(G)]
        d_idx = [torch.from_numpy(m[0]).cuda() for m in mats]
        d_sc = [torch.from_numpy(m[1].view(np.int16)).cuda() for m in mats]
        d_x = torch.from_numpy(synth.activations(8, N, T=G)).cuda()
        y = torch.empty((G, M), dtype=torch.float32, device="cuda")
        wb.init(0)
        wb.codebooks_load_f16(synth.codebooks(rng, 3))
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        wb.vq_matvec_dev_noalloc([t.data_ptr() for t in d_idx], [t.data_ptr() for t in d_sc],
                                 [d_x[g].data_ptr() for g in range(G)],
                                 [y[g].data_ptr() for g in range(G)], M, N, 0, 3, 0)
        torch.cuda.synchronize()
        free1 = torch.cuda.mem_get_info()[0]
        assert wb.device_errors() == 0
        assert np.isfinite(y.cpu().numpy()).all()
        print("TAKEN", free0 - free1)
    """ % root)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    taken = int(r.stdout.split("TAKEN")[-1].split()[0])
    assert taken < (2 << 20), f"the first call after init took {taken} bytes of device memory"
