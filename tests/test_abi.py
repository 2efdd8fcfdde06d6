"""The C-ABI library, without touching a GPU: it builds for sm_100a, exports
every entry point include/waste_cuda.h declares, and declines cleanly when no
sm_100 device is present (the reference's registration contract,
src/waste_backend.h:116-120: return NULL, keep the previous backend)."""
import ctypes as C
import os
import re
import subprocess

import pytest

import warp_b200 as wb
from warp_b200 import build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "waste_cuda.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    src = re.sub(r"typedef struct \{.*?\}\s*\w+;", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(waste_\w+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib_path():
    return build.build()


def test_exports_match_header(lib_path):
    names = declared_functions()
    assert len(names) >= 15
    out = subprocess.run(["nm", "-D", "--defined-only", lib_path], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\sT\s(\w+)$", out, flags=re.M))
    missing = [n for n in names if n not in exported]
    assert not missing, missing
    assert sorted(wb.EXPORTS) == names


def test_library_is_built_for_sm100a_only():
    """Every nvcc step of warp_b200/build.py compiles real sm_100a code and no
    other target (no PTX for a JIT to pick up elsewhere)."""
    assert build.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]
    src = open(build.__file__).read()
    assert set(re.findall(r"compute_(\w+)", src)) == {"100a"}
    assert set(re.findall(r"\bsm_(\w+)", src)) == {"100a"}
    assert src.count("*ARCH") == src.count("[NVCC,")


@pytest.mark.gpu
def test_kernels_run_as_sm100_binaries(lib_path):
    """On the device: the loaded kernels are sm_100 machine code
    (cudaFuncGetAttributes binaryVersion)."""
    import warp_b200 as w
    w.init(0)
    lib = w.load_library()
    lib.wc_binary_version.restype = C.c_int
    assert lib.wc_binary_version() == 100


def _has_device():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.mark.skipif(_has_device(), reason="declining is only observable without a device")
def test_declines_without_device(lib_path):
    lib = wb.load_library()
    assert lib.waste_register_cuda(None) is None
    assert lib.waste_cuda_init(0) == wb.E_NODEV
    assert b"device" in lib.waste_cuda_last_error()
    slots = wb.VqSlots()
    assert lib.waste_register_cuda_vq(C.byref(slots)) == wb.E_NODEV
    assert not slots.moe_experts


def test_argument_checks_need_no_device(lib_path):
    lib = wb.load_library()
    assert lib.waste_cuda_vq_bank_load(-1, 1, 4096, 0, 1, None, 8, 8, 3) == wb.E_ARG
    assert lib.waste_cuda_codebooks_load(None, 1, 256, 8) == wb.E_ARG
    assert lib.waste_cuda_codebooks_load_f16(None, 1, 128, 8) == wb.E_ARG
    assert lib.waste_cuda_moe_experts(None) == wb.E_ARG


def test_slot_table_layout_matches_header():
    """The ctypes mirror of waste_vq_slots has the header's fields in order
    (a shorter mirror would be overrun by waste_register_cuda_vq)."""
    src = open(HEADER).read()
    body = src[src.index("typedef struct {\n    int  (*codebooks_load)"):]
    body = body[:body.index("} waste_vq_slots;")]
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
    fields = re.findall(r"\(\*(\w+)\)", body)
    assert [f[0] for f in wb.VqSlots._fields_] == fields
