"""warp_b200 — B200 (sm_100a) backend for WARP's VQ3R routed-expert FFN.

The product is the C-ABI library ``warp_b200/lib/libwaste_cuda.so``
(include/waste_cuda.h). This module binds it with ctypes so tests and the
benchmark call exactly the entry points the reference engine's integration
calls. There is no fallback: if the library is missing or no sm_100 device is
present, calls raise.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libwaste_cuda.so")

# Entry points declared in include/waste_cuda.h, in header order.
EXPORTS = (
    "waste_register_cuda", "waste_register_cuda_vq",
    "waste_cuda_init", "waste_cuda_shutdown", "waste_cuda_device",
    "waste_cuda_last_error", "waste_cuda_backend_name",
    "waste_cuda_codebooks_load", "waste_cuda_codebooks_load_f16",
    "waste_cuda_vq_bank_load", "waste_cuda_vq_bank_free",
    "waste_cuda_moe_trunk_load", "waste_cuda_moe_experts",
    "waste_cuda_moe_chunk_experts", "waste_cuda_moe_layer",
    "waste_cuda_moe_layer_dev", "waste_cuda_lutb", "waste_cuda_vq_matvec",
    "waste_cuda_vq_dequant", "waste_cuda_vq_matvec_dev",
    "waste_cuda_launch_count", "waste_cuda_profile", "waste_cuda_profile_read",
    "waste_cuda_device_errors", "waste_cuda_vq_matvec_dev_noalloc",
    "waste_cuda_vq_bank_reserve", "waste_cuda_moe_layer_part_dev",
    "waste_cuda_ep_range", "waste_cuda_ep_unique_id", "waste_cuda_ep_init",
    "waste_cuda_ep_shutdown", "waste_cuda_ep_moe_layer_dev", "waste_cuda_moe_prefill_dev",
    "waste_cuda_ep_moe_layer_rep_dev", "waste_cuda_moe_norm_load", "waste_cuda_moe_block",
    "waste_cuda_moe_block_dev", "waste_cuda_ep_moe_block_dev", "waste_cuda_ep_moe_block_rep_dev",
    "waste_cuda_moe_activation", "waste_cuda_mvq_rows_dev", "waste_cuda_release_host_buffers",
    "waste_cuda_vq_sel_bytes", "waste_cuda_vq_sel_build_dev", "waste_cuda_vq_matvec_sel_dev",
    "waste_cuda_vq_bank_load_file", "waste_cuda_vq4p_matvec", "waste_cuda_vq4p_matvec_dev",
    "waste_cuda_vq4p_table", "waste_cuda_kda_step", "waste_cuda_short_conv_step",
    "waste_cuda_rmsnorm_gated_heads", "waste_cuda_state_push", "waste_cuda_state_pull",
    "waste_cuda_kda_step_dev", "waste_cuda_short_conv_dev", "waste_cuda_rmsnorm_gated_dev",
    "waste_cuda_vq_encode", "waste_cuda_vq_encode_dev", "waste_cuda_vq_lloyd",
    "waste_cuda_vq_lloyd_dev", "waste_cuda_kda_layer", "waste_cuda_mla_layer",
)

PHASES = ("router", "act", "gateup", "down", "combine", "matvec", "matvec_reduce", "ep_publish",
          "ep_finalize")

OK, E_ARG, E_DEVICE, E_RECORD, E_NOBANK, E_NOMEM, E_NODEV = 0, -1, -2, -3, -4, -5, -6
DERR_ROUTE_WAIT, DERR_TMA_WAIT, DERR_BAD_EXPERT, DERR_PEER_WAIT = 1, 2, 4, 8


class WasteCudaError(RuntimeError):
    def __init__(self, rc: int, msg: str):
        super().__init__(f"waste_cuda status {rc}: {msg}")
        self.rc = rc


class MoeCall(C.Structure):
    """struct waste_moe_call (include/waste_cuda.h)."""
    _fields_ = [("layer", C.c_int), ("K", C.c_int),
                ("idx", C.POINTER(C.c_int)), ("w", C.POINTER(C.c_float)),
                ("x", C.POINTER(C.c_float)), ("ysum", C.POINTER(C.c_float)),
                ("lat", C.c_int), ("inter", C.c_int), ("act", C.c_int),
                ("situ_beta", C.c_float), ("situ_linear_beta", C.c_float)]


class MoeChunkCall(C.Structure):
    """struct waste_moe_chunk_call (include/waste_cuda.h)."""
    _fields_ = [("layer", C.c_int), ("nT", C.c_int), ("K", C.c_int),
                ("route", C.POINTER(C.c_int)), ("rw", C.POINTER(C.c_float)),
                ("x", C.POINTER(C.c_float)), ("ysum", C.POINTER(C.c_float)),
                ("lat", C.c_int), ("inter", C.c_int), ("act", C.c_int),
                ("situ_beta", C.c_float), ("situ_linear_beta", C.c_float)]


class VqSlots(C.Structure):
    """waste_vq_slots: the expert-path slots next to waste_kernels."""
    _fields_ = [("codebooks_load", C.c_void_p), ("vq_bank_load", C.c_void_p),
                ("vq_bank_free", C.c_void_p), ("moe_experts", C.c_void_p),
                ("moe_chunk_experts", C.c_void_p), ("vq_bank_load_file", C.c_void_p),
                ("state_push", C.c_void_p), ("state_pull", C.c_void_p),
                ("rmsnorm_gated_heads", C.c_void_p), ("moe_trunk_load", C.c_void_p),
                ("moe_activation", C.c_void_p), ("moe_layer", C.c_void_p),
                ("kda_layer", C.c_void_p), ("mla_layer", C.c_void_p)]


_lib = None


def library_path() -> str:
    return LIB_PATH


def load_library() -> C.CDLL:
    """Load libwaste_cuda.so (built in-tree by warp_b200.build)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise FileNotFoundError(
            f"{LIB_PATH} is missing: run `python -c 'import __graft_entry__ as g; g.build()'`")
    lib = C.CDLL(LIB_PATH)
    P = C.c_void_p
    f32p, i32p = C.POINTER(C.c_float), C.POINTER(C.c_int)
    sig = {
        "waste_register_cuda": (C.c_char_p, [P]),
        "waste_register_cuda_vq": (C.c_int, [C.POINTER(VqSlots)]),
        "waste_cuda_init": (C.c_int, [C.c_int]),
        "waste_cuda_shutdown": (None, []),
        "waste_cuda_device": (C.c_int, []),
        "waste_cuda_last_error": (C.c_char_p, []),
        "waste_cuda_backend_name": (C.c_char_p, []),
        "waste_cuda_codebooks_load": (C.c_int, [P, C.c_int, C.c_int, C.c_int]),
        "waste_cuda_codebooks_load_f16": (C.c_int, [P, C.c_int, C.c_int, C.c_int]),
        "waste_cuda_vq_bank_load": (C.c_int, [C.c_int, C.c_int, C.c_size_t, C.c_int, C.c_int,
                                              P, C.c_int, C.c_int, C.c_int]),
        "waste_cuda_vq_bank_free": (None, [C.c_int]),
        "waste_cuda_moe_trunk_load": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                                C.c_float, P, P, C.c_int, P, P, P, P, P, P]),
        "waste_cuda_moe_experts": (C.c_int, [C.POINTER(MoeCall)]),
        "waste_cuda_moe_chunk_experts": (C.c_int, [C.POINTER(MoeChunkCall)]),
        "waste_cuda_moe_layer": (C.c_int, [C.c_int, P, P, P, P]),
        "waste_cuda_moe_layer_dev": (C.c_int, [C.c_int, P, P, P, P, P]),
        "waste_cuda_lutb": (C.c_int, [P, P, C.c_int, C.c_int, C.c_int]),
        "waste_cuda_vq_matvec": (C.c_int, [P, P, P, P, C.c_int, C.c_int, C.c_int, C.c_int]),
        "waste_cuda_vq_dequant": (C.c_int, [P, P, P, C.c_int, C.c_int, C.c_int, C.c_int]),
        "waste_cuda_vq_matvec_dev": (C.c_int, [C.c_int, P, P, P, P, C.c_int, C.c_int,
                                               C.c_int, C.c_int, P]),
        "waste_cuda_vq_matvec_dev_noalloc": (C.c_int, [C.c_int, P, P, P, P, C.c_int,
                                                       C.c_int, C.c_int, C.c_int, P]),
        "waste_cuda_launch_count": (C.c_uint64, []),
        "waste_cuda_profile": (C.c_int, [C.c_int]),
        "waste_cuda_profile_read": (C.c_int, [P, P, C.c_int]),
        "waste_cuda_device_errors": (C.c_uint, []),
        "waste_cuda_vq_bank_reserve": (C.c_int, [C.c_int, C.c_int, C.c_size_t, C.c_int, C.c_int,
                                                 C.c_int, C.c_int, C.c_int]),
        "waste_cuda_moe_layer_part_dev": (C.c_int, [C.c_int, C.c_int, P, P, C.c_int, C.c_int,
                                                    P, P, P]),
        "waste_cuda_ep_range": (C.c_int, [C.c_int, C.c_int, C.c_int, P, P]),
        "waste_cuda_ep_unique_id": (C.c_int, [P, C.c_size_t]),
        "waste_cuda_ep_init": (C.c_int, [C.c_int, C.c_int, P, C.c_size_t]),
        "waste_cuda_ep_shutdown": (None, []),
        "waste_cuda_ep_moe_layer_dev": (C.c_int, [C.c_int, C.c_int, P, P, P, P, P]),
        "waste_cuda_ep_moe_layer_rep_dev": (C.c_int, [C.c_int, C.c_int, P, P, P, P, P]),
        "waste_cuda_moe_prefill_dev": (C.c_int, [C.c_int, C.c_int, C.c_int, P, P, P, P, P]),
        "waste_cuda_moe_norm_load": (C.c_int, [C.c_int, C.c_int, P, C.c_float]),
        "waste_cuda_moe_activation": (C.c_int, [C.c_int, C.c_int, C.c_float, C.c_float]),
        "waste_cuda_mvq_rows_dev": (C.c_int, [P, P, P, P, C.c_int, C.c_int, C.c_int, C.c_int,
                                              C.c_int, C.c_size_t, P]),
        "waste_cuda_release_host_buffers": (None, []),
        "waste_cuda_vq_sel_bytes": (C.c_size_t, [C.c_int, C.c_int, C.c_int, C.c_int]),
        "waste_cuda_vq_bank_load_file": (C.c_int, [C.c_int, C.c_int, C.c_int64, C.c_int,
                                                   C.c_size_t, C.c_int, C.c_int, C.c_int,
                                                   C.c_int, C.c_int]),
        "waste_cuda_vq_sel_build_dev": (C.c_int, [P, P, C.c_int, C.c_int, C.c_int, C.c_int, P]),
        "waste_cuda_vq_matvec_sel_dev": (C.c_int, [C.c_int, P, P, P, P, P, C.c_int, C.c_int,
                                                   C.c_int, C.c_int, C.c_int, P]),
        "waste_cuda_moe_block": (C.c_int, [C.c_int, P, P, P, P]),
        "waste_cuda_moe_block_dev": (C.c_int, [C.c_int, C.c_int, P, P, P, P, P]),
        "waste_cuda_ep_moe_block_dev": (C.c_int, [C.c_int, C.c_int, P, P, P, P, P]),
        "waste_cuda_ep_moe_block_rep_dev": (C.c_int, [C.c_int, C.c_int, P, P, P, P, P]),
        "waste_cuda_vq4p_matvec": (C.c_int, [P, P, P, P, C.c_int, C.c_int, C.c_int]),
        "waste_cuda_vq4p_matvec_dev": (C.c_int, [C.c_int, P, P, P, P, C.c_int, C.c_int,
                                                 C.c_int, P]),
        "waste_cuda_vq4p_table": (C.c_int, [P, P, P, C.c_int, C.c_int]),
        "waste_cuda_kda_step": (C.c_int, [C.c_int, C.c_int, C.c_int, P, P, P, P, P, P, P]),
        "waste_cuda_short_conv_step": (C.c_int, [C.c_int, C.c_int, P, P, P, P, P]),
        "waste_cuda_rmsnorm_gated_heads": (C.c_int, [C.c_int, C.c_int, P, P, P, C.c_float, P]),
        "waste_cuda_state_push": (C.c_int, [P, C.c_size_t]),
        "waste_cuda_state_pull": (C.c_int, [P, C.c_size_t]),
        "waste_cuda_kda_step_dev": (C.c_int, [C.c_int, C.c_int, C.c_int, P, P, P, P, P, P, P, P]),
        "waste_cuda_short_conv_dev": (C.c_int, [C.c_int, C.c_int, P, P, P, P, P, P]),
        "waste_cuda_rmsnorm_gated_dev": (C.c_int, [C.c_int, C.c_int, P, P, P, C.c_float, P, P]),
        "waste_cuda_vq_encode": (C.c_int, [P, C.c_int, P, C.c_int, C.c_int, C.c_int, P]),
        "waste_cuda_vq_encode_dev": (C.c_int, [P, C.c_int, P, C.c_int, C.c_int, C.c_int, P, P]),
        "waste_cuda_vq_lloyd": (C.c_int, [P, C.c_int, P, C.c_int, C.c_int]),
        "waste_cuda_vq_lloyd_dev": (C.c_int, [P, C.c_int, P, C.c_int, C.c_int, P, P]),
        "waste_cuda_kda_layer": (C.c_int, [P, P, P]),
        "waste_cuda_mla_layer": (C.c_int, [P, C.c_int, P, P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    del f32p, i32p
    _lib = lib
    return lib


def _ptr(a: np.ndarray) -> C.c_void_p:
    return C.c_void_p(a.ctypes.data)


def _check(rc: int):
    if rc != 0:
        msg = load_library().waste_cuda_last_error()
        raise WasteCudaError(rc, msg.decode() if msg else "(no message)")


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def init(device: int = -1) -> str:
    lib = load_library()
    _check(lib.waste_cuda_init(device))
    return lib.waste_cuda_backend_name().decode()


def shutdown():
    load_library().waste_cuda_shutdown()


def register_cuda() -> str | None:
    """waste_register_cuda: the backend name, or None when it declines."""
    n = load_library().waste_register_cuda(None)
    return n.decode() if n else None


def register_cuda_vq() -> VqSlots:
    s = VqSlots()
    _check(load_library().waste_register_cuda_vq(C.byref(s)))
    return s


def device_errors() -> int:
    """Sticky device error bits (WASTE_CUDA_DERR_*); reading clears them."""
    return int(load_library().waste_cuda_device_errors())


def launch_count() -> int:
    return int(load_library().waste_cuda_launch_count())


def profile(on: bool):
    """Phase timers on/off (CUDA events around every kernel launch)."""
    _check(load_library().waste_cuda_profile(1 if on else 0))


def profile_read() -> dict:
    """{phase: (total ms, launches)} since the last read; resets."""
    n = len(PHASES)
    ms = np.zeros(n, dtype=np.float64)
    cnt = np.zeros(n, dtype=np.uint64)
    _check(load_library().waste_cuda_profile_read(_ptr(ms), _ptr(cnt), n))
    return {p: (float(ms[i]), int(cnt[i])) for i, p in enumerate(PHASES)}


def codebooks_load(books: np.ndarray):
    b = _f32(books)
    _check(load_library().waste_cuda_codebooks_load(_ptr(b), b.shape[0], b.shape[1], b.shape[2]))


def codebooks_load_f16(raw: np.ndarray):
    r = np.ascontiguousarray(raw, dtype=np.uint16)
    _check(load_library().waste_cuda_codebooks_load_f16(_ptr(r), r.shape[0], r.shape[1],
                                                        r.shape[2]))


def vq_bank_load(layer: int, n_experts: int, rec_bytes: int, first: int, count: int,
                 records: np.ndarray, inter: int, lat: int, stages: int = 3):
    r = np.ascontiguousarray(records, dtype=np.uint8)
    if r.size < count * rec_bytes:
        raise ValueError("records buffer shorter than count * rec_bytes")
    _check(load_library().waste_cuda_vq_bank_load(layer, n_experts, rec_bytes, first, count,
                                                  _ptr(r), inter, lat, stages))


def vq_bank_load_file(layer: int, path: str, n_experts: int, rec_bytes: int, first: int,
                      count: int, inter: int, lat: int, stages: int = 3, offset: int = 0):
    """Records [first, first+count) of a layer straight from a bank file."""
    fd = os.open(path, os.O_RDONLY)
    try:
        _check(load_library().waste_cuda_vq_bank_load_file(layer, fd, offset, n_experts,
                                                           rec_bytes, first, count, inter, lat,
                                                           stages))
    finally:
        os.close(fd)


def vq_bank_free(layer: int):
    load_library().waste_cuda_vq_bank_free(layer)


def vq_bank_reserve(layer: int, n_experts: int, rec_bytes: int, first: int, count: int,
                    inter: int, lat: int, stages: int = 3):
    """HBM for records [first, first+count) of a layer, ahead of loading."""
    _check(load_library().waste_cuda_vq_bank_reserve(layer, n_experts, rec_bytes, first, count,
                                                     inter, lat, stages))


def moe_trunk_load(layer: int, n_experts: int, hidden: int, top_k: int, renorm: int,
                   routed_scale: float, router: np.ndarray, bias: np.ndarray | None,
                   sh_inter: int = 0, sh: dict | None = None):
    rt = _f32(router)
    b = _f32(bias) if bias is not None else None
    keep = [rt, b]
    ptrs = []
    if sh_inter:
        for k in ("gate", "up", "down"):
            q = np.ascontiguousarray(sh[k][0], dtype=np.int8)
            s = np.ascontiguousarray(sh[k][1], dtype=np.uint16)
            keep += [q, s]
            ptrs += [_ptr(q), _ptr(s)]
    else:
        ptrs = [None] * 6
    _check(load_library().waste_cuda_moe_trunk_load(
        layer, n_experts, hidden, top_k, renorm, C.c_float(routed_scale), _ptr(rt),
        _ptr(b) if b is not None else None, sh_inter, *ptrs))
    del keep


def load_layer(L, trunk: bool = True):
    """Codebooks, the whole bank and (optionally) the trunk of a synth.MoELayer,
    with its activation."""
    codebooks_load_f16(L.books_raw)
    vq_bank_load(L.layer, L.n_experts, L.rec_bytes, 0, L.n_experts, L.bank, L.inter,
                 L.hidden, L.stages)
    if trunk:
        moe_trunk_load(L.layer, L.n_experts, L.hidden, L.top_k, L.renorm, L.routed_scale,
                       L.router, L.bias, L.shared_inter, L.sh)
    moe_activation(L.layer, int(getattr(L, "act_situ", 0)), float(getattr(L, "situ_beta", 0.0)),
                   float(getattr(L, "situ_lbeta", 0.0)))


def moe_experts(layer: int, idx, w, x, lat: int, inter: int, act: int = 0,
                situ_beta: float = 0.0, situ_lbeta: float = 0.0) -> np.ndarray:
    """The expert loop for one token (waste_moe_call): ysum[lat]."""
    i = np.ascontiguousarray(idx, dtype=np.int32)
    ww = _f32(w)
    xx = _f32(x)
    y = np.empty(lat, dtype=np.float32)
    c = MoeCall(layer, i.size, i.ctypes.data_as(C.POINTER(C.c_int)),
                ww.ctypes.data_as(C.POINTER(C.c_float)), xx.ctypes.data_as(C.POINTER(C.c_float)),
                y.ctypes.data_as(C.POINTER(C.c_float)), lat, inter, act, situ_beta, situ_lbeta)
    _check(load_library().waste_cuda_moe_experts(C.byref(c)))
    return y


def moe_chunk_experts(layer: int, route, rw, x, lat: int, inter: int, act: int = 0,
                      situ_beta: float = 0.0, situ_lbeta: float = 0.0) -> np.ndarray:
    """The prefill expert loop (waste_moe_chunk_call): ysum[nT][lat]."""
    r = np.ascontiguousarray(route, dtype=np.int32)
    ww = _f32(rw)
    xx = _f32(x)
    nT, K = r.shape
    y = np.empty((nT, lat), dtype=np.float32)
    c = MoeChunkCall(layer, nT, K, r.ctypes.data_as(C.POINTER(C.c_int)),
                     ww.ctypes.data_as(C.POINTER(C.c_float)),
                     xx.ctypes.data_as(C.POINTER(C.c_float)),
                     y.ctypes.data_as(C.POINTER(C.c_float)), lat, inter, act, situ_beta,
                     situ_lbeta)
    _check(load_library().waste_cuda_moe_chunk_experts(C.byref(c)))
    return y


def moe_layer(layer: int, x, K: int, hidden: int):
    """Whole layer on host buffers: (out[hidden], idx[K], w[K])."""
    xx = _f32(x)
    out = np.empty(hidden, dtype=np.float32)
    idx = np.empty(K, dtype=np.int32)
    w = np.empty(K, dtype=np.float32)
    _check(load_library().waste_cuda_moe_layer(layer, _ptr(xx), _ptr(out), _ptr(idx), _ptr(w)))
    return out, idx, w


def moe_layer_dev(layer: int, d_x: int, d_out: int, d_idx: int, d_w: int, stream: int = 0):
    _check(load_library().waste_cuda_moe_layer_dev(layer, C.c_void_p(d_x), C.c_void_p(d_out),
                                                   C.c_void_p(d_idx), C.c_void_p(d_w),
                                                   C.c_void_p(stream or None)))


def moe_activation(layer: int, act: int, situ_beta: float = 0.0, situ_lbeta: float = 0.0):
    """The layer's gated activation on the device-routed paths (0 SiLU, 1 SiTU)."""
    _check(load_library().waste_cuda_moe_activation(layer, act, C.c_float(situ_beta),
                                                    C.c_float(situ_lbeta)))


def moe_norm_load(layer: int, norm_w, eps: float):
    """The layer's post-attention rmsnorm weight for the MoE block."""
    w = _f32(norm_w)
    _check(load_library().waste_cuda_moe_norm_load(layer, w.size, _ptr(w), C.c_float(eps)))


def moe_block(layer: int, h, K: int, hidden: int):
    """h + moe_layer(rmsnorm(h)) on host buffers: (h_out[hidden], idx[K], w[K])."""
    hh = _f32(h)
    out = np.empty(hidden, dtype=np.float32)
    idx = np.empty(K, dtype=np.int32)
    w = np.empty(K, dtype=np.float32)
    _check(load_library().waste_cuda_moe_block(layer, _ptr(hh), _ptr(out), _ptr(idx), _ptr(w)))
    return out, idx, w


def moe_block_dev(layer: int, T: int, d_h: int, d_out: int, d_idx: int, d_w: int,
                  stream: int = 0):
    """T tokens' h + moe_layer(rmsnorm(h)), device pointers."""
    v = lambda p: C.c_void_p(int(p) or None)
    _check(load_library().waste_cuda_moe_block_dev(layer, T, v(d_h), v(d_out), v(d_idx), v(d_w),
                                                   v(stream)))


def moe_layer_part_dev(layer: int, T: int, d_x: int, d_out: int, sh_t0: int, sh_t1: int,
                       d_idx: int, d_w: int, stream: int = 0):
    """The experts this device holds (+ the shared expert for tokens
    [sh_t0, sh_t1)) for T tokens: partial sums to be added over devices."""
    v = lambda p: C.c_void_p(int(p) or None)
    _check(load_library().waste_cuda_moe_layer_part_dev(layer, T, v(d_x), v(d_out), sh_t0, sh_t1,
                                                        v(d_idx), v(d_w), v(stream)))


def moe_prefill_dev(layer: int, T: int, K: int, d_route: int, d_rw: int, d_x: int, d_out: int,
                    stream: int = 0):
    """Prefill expert loop on the tensor cores (device pointers)."""
    v = lambda p: C.c_void_p(int(p) or None)
    _check(load_library().waste_cuda_moe_prefill_dev(layer, T, K, v(d_route), v(d_rw), v(d_x),
                                                     v(d_out), v(stream)))


def mvq_rows_dev(d_y: int, d_W: int, d_ws: int, d_x: int, r0: int, r1: int, inp: int,
                 group: int, bits: int, rowbytes: int, stream: int = 0):
    """The trunk matvec (mvq_rows_f32) on device pointers."""
    v = lambda p: C.c_void_p(int(p) or None)
    _check(load_library().waste_cuda_mvq_rows_dev(v(d_y), v(d_W), v(d_ws), v(d_x), r0, r1, inp,
                                                  group, bits, rowbytes, v(stream)))


def lutb(x, cb_base: int, stages: int = 3) -> np.ndarray:
    xx = _f32(x)
    nv = xx.size // 8
    lut = np.empty((nv, stages, 256), dtype=np.float32)
    _check(load_library().waste_cuda_lutb(_ptr(lut), _ptr(xx), cb_base, nv, stages))
    return lut


def vq_matvec(idx, scale, x, M: int, N: int, cb_base: int, stages: int = 3) -> np.ndarray:
    i = np.ascontiguousarray(idx, dtype=np.uint8)
    s = np.ascontiguousarray(scale, dtype=np.uint16)
    xx = _f32(x)
    y = np.empty(M, dtype=np.float32)
    _check(load_library().waste_cuda_vq_matvec(_ptr(y), _ptr(i), _ptr(s), _ptr(xx), M, N,
                                               cb_base, stages))
    return y


def vq_dequant(idx, scale, M: int, N: int, cb_base: int, stages: int = 3) -> np.ndarray:
    i = np.ascontiguousarray(idx, dtype=np.uint8)
    s = np.ascontiguousarray(scale, dtype=np.uint16)
    W = np.empty((M, N), dtype=np.float32)
    _check(load_library().waste_cuda_vq_dequant(_ptr(W), _ptr(i), _ptr(s), M, N, cb_base,
                                                stages))
    return W


def vq_matvec_dev(idx_ptrs, scale_ptrs, x_ptrs, y_ptrs, M: int, N: int, cb_base: int,
                  stages: int = 3, stream: int = 0):
    G = len(idx_ptrs)
    arr = lambda v: (C.c_void_p * G)(*[C.c_void_p(int(p)) for p in v])
    _check(load_library().waste_cuda_vq_matvec_dev(
        G, arr(idx_ptrs), arr(scale_ptrs), arr(x_ptrs), arr(y_ptrs), M, N, cb_base, stages,
        C.c_void_p(stream or None)))


def vq_sel_bytes(M: int, N: int, stages: int = 3, copies: int = 2) -> int:
    return int(load_library().waste_cuda_vq_sel_bytes(M, N, stages, copies))


def vq_sel_build_dev(d_idx: int, d_sel: int, M: int, N: int, stages: int = 3, copies: int = 2,
                     stream: int = 0):
    """Writes a matrix's copy-select stream (device pointers)."""
    _check(load_library().waste_cuda_vq_sel_build_dev(C.c_void_p(d_idx), C.c_void_p(d_sel), M, N,
                                                      stages, copies, C.c_void_p(stream or None)))


def vq_matvec_sel_dev(idx_ptrs, sel_ptrs, scale_ptrs, x_ptrs, y_ptrs, M: int, N: int,
                      cb_base: int, stages: int = 3, copies: int = 2, stream: int = 0):
    """vq_matvec_dev with interleaved table copies and copy-select streams."""
    G = len(idx_ptrs)
    arr = lambda v: (C.c_void_p * G)(*[C.c_void_p(int(p)) for p in v])
    _check(load_library().waste_cuda_vq_matvec_sel_dev(
        G, arr(idx_ptrs), arr(sel_ptrs), arr(scale_ptrs), arr(x_ptrs), arr(y_ptrs), M, N, cb_base,
        stages, copies, C.c_void_p(stream or None)))


NOALLOC_SCRATCH_BYTES = 32 << 20


def vq_matvec_dev_noalloc(idx_ptrs, scale_ptrs, x_ptrs, y_ptrs, M: int, N: int, cb_base: int,
                          stages: int = 3, stream: int = 0):
    """vq_matvec_dev without any device allocation: for callers that reserved
    the device's memory up front, or cannot take cudaFree's device-wide
    synchronisation mid-run. Partial sums use a fixed 32 MiB array built
    into the library (G * ceil(N/64) * M * 4 bytes at most; larger calls
    raise). The array is taken when init binds the device, so no call after
    init allocates; calls overlapping on the GPU race on that array."""
    G = len(idx_ptrs)
    arr = lambda v: (C.c_void_p * G)(*[C.c_void_p(int(p)) for p in v])
    _check(load_library().waste_cuda_vq_matvec_dev_noalloc(
        G, arr(idx_ptrs), arr(scale_ptrs), arr(x_ptrs), arr(y_ptrs), M, N, cb_base, stages,
        C.c_void_p(stream or None)))


def vq4p_matvec(idx, scale, x, M: int, N: int, cb_base: int) -> np.ndarray:
    """y = VQ4P(idx, scale) . x (64-entry codebooks loaded; host buffers)."""
    i = np.ascontiguousarray(idx, dtype=np.uint8)
    s = np.ascontiguousarray(scale, dtype=np.uint16)
    xx = _f32(x)
    y = np.empty(M, dtype=np.float32)
    _check(load_library().waste_cuda_vq4p_matvec(_ptr(y), _ptr(i), _ptr(s), _ptr(xx), M, N,
                                                 cb_base))
    return y


def vq4p_matvec_dev(idx_ptrs, scale_ptrs, x_ptrs, y_ptrs, M: int, N: int, cb_base: int,
                    stream: int = 0):
    """G VQ4P matvecs of one shape on device pointers."""
    G = len(idx_ptrs)
    arr = lambda v: (C.c_void_p * G)(*[C.c_void_p(int(p)) for p in v])
    _check(load_library().waste_cuda_vq4p_matvec_dev(
        G, arr(idx_ptrs), arr(scale_ptrs), arr(x_ptrs), arr(y_ptrs), M, N, cb_base,
        C.c_void_p(stream or None)))


def vq4p_table(x, cb_base: int):
    """The int8 tables of x (q [N/8][4][64]) and their scales (one per 32
    positions)."""
    xx = _f32(x)
    nv = xx.size // 8
    q = np.empty((nv, 4, 64), dtype=np.int8)
    qs = np.empty((nv + 31) // 32, dtype=np.float32)
    _check(load_library().waste_cuda_vq4p_table(_ptr(q), _ptr(qs), _ptr(xx), xx.size, cb_base))
    return q, qs

# ---- KDA ----------------------------------------------------------------------

def kda_step(H: int, K: int, V: int, q, k, v, g_log, beta, S: np.ndarray) -> np.ndarray:
    """One decode step (the kda_step slot): S, a float32 array the caller
    keeps, is held in HBM from the first call on (its host bytes are stale
    until state_pull). Returns o [H*V]."""
    a = [_f32(t) for t in (q, k, v, g_log, beta)]
    assert S.dtype == np.float32 and S.flags.c_contiguous
    o = np.empty(H * V, dtype=np.float32)
    _check(load_library().waste_cuda_kda_step(H, K, V, *[_ptr(t) for t in a], _ptr(S), _ptr(o)))
    return o


def short_conv_step(C_: int, KS: int, w, bias, ring: np.ndarray, x) -> np.ndarray:
    """The short_conv_step slot: ring (float32, caller-kept) held in HBM."""
    ww = _f32(w)
    assert ring.dtype == np.float32 and ring.flags.c_contiguous
    bb = _f32(bias) if bias is not None else None
    xx = _f32(x)
    y = np.empty(C_, dtype=np.float32)
    _check(load_library().waste_cuda_short_conv_step(C_, KS, _ptr(ww), _ptr(bb) if bb is not None
                                                     else None, _ptr(ring), _ptr(xx), _ptr(y)))
    return y


def rmsnorm_gated_heads(nh: int, C_: int, x, gate, w, eps: float) -> np.ndarray:
    xx, gg, ww = _f32(x), _f32(gate), _f32(w)
    y = np.empty(nh * C_, dtype=np.float32)
    _check(load_library().waste_cuda_rmsnorm_gated_heads(nh, C_, _ptr(xx), _ptr(gg), _ptr(ww),
                                                         C.c_float(eps), _ptr(y)))
    return y


def state_pull(a: np.ndarray):
    _check(load_library().waste_cuda_state_pull(_ptr(a), a.nbytes))


def state_push(a: np.ndarray):
    _check(load_library().waste_cuda_state_push(_ptr(a), a.nbytes))


def kda_step_dev(H, K, V, d_q, d_k, d_v, d_g, d_beta, d_S, d_o, stream: int = 0):
    v = lambda p: C.c_void_p(int(p)) if p else None
    _check(load_library().waste_cuda_kda_step_dev(H, K, V, v(d_q), v(d_k), v(d_v), v(d_g),
                                                  v(d_beta), v(d_S), v(d_o), v(stream)))


def short_conv_dev(C_, KS, d_w, d_bias, d_ring, d_x, d_y, stream: int = 0):
    v = lambda p: C.c_void_p(int(p)) if p else None
    _check(load_library().waste_cuda_short_conv_dev(C_, KS, v(d_w), v(d_bias), v(d_ring), v(d_x),
                                                    v(d_y), v(stream)))


def rmsnorm_gated_dev(nh, C_, d_x, d_gate, d_w, eps, d_y, stream: int = 0):
    v = lambda p: C.c_void_p(int(p)) if p else None
    _check(load_library().waste_cuda_rmsnorm_gated_dev(nh, C_, v(d_x), v(d_gate), v(d_w),
                                                       C.c_float(eps), v(d_y), v(stream)))


def release_host_buffers():
    """Drop every device copy keyed by a host address (trunk mirrors, KDA
    state and weights): what the engine calls before freeing a model."""
    load_library().waste_cuda_release_host_buffers()


# ---- the converter's RVQ encoder ------------------------------------------------

def vq_encode(X, books) -> np.ndarray:
    """X [n][dim], books [stages][entries][dim] -> codes [n][stages] uint8."""
    xx = np.ascontiguousarray(X, dtype=np.float32)
    bb = np.ascontiguousarray(books, dtype=np.float32)
    n, dim = xx.shape
    stages, entries = bb.shape[0], bb.shape[1]
    out = np.empty((n, stages), dtype=np.uint8)
    _check(load_library().waste_cuda_vq_encode(_ptr(xx), n, _ptr(bb), stages, entries, dim,
                                               _ptr(out)))
    return out


def vq_lloyd(X, C):
    """One Lloyd iteration: returns (new centroids, non-empty clusters)."""
    xx = np.ascontiguousarray(X, dtype=np.float32)
    cc = np.array(C, dtype=np.float32, copy=True, order="C")
    rc = load_library().waste_cuda_vq_lloyd(_ptr(xx), xx.shape[0], _ptr(cc), cc.shape[0],
                                            cc.shape[1])
    if rc < 0:
        _check(rc)
    return cc, rc


def vq_encode_dev(d_X, n, d_books, stages, entries, dim, d_out, stream: int = 0):
    v = lambda p: C.c_void_p(int(p)) if p else None
    _check(load_library().waste_cuda_vq_encode_dev(v(d_X), n, v(d_books), stages, entries, dim,
                                                   v(d_out), v(stream)))


def vq_lloyd_dev(d_X, n, d_C, entries, dim, d_live, stream: int = 0):
    v = lambda p: C.c_void_p(int(p)) if p else None
    _check(load_library().waste_cuda_vq_lloyd_dev(v(d_X), n, v(d_C), entries, dim, v(d_live),
                                                  v(stream)))
