"""ctypes bindings for the parity checker. TEST INFRASTRUCTURE ONLY.

Two libraries, both built by oracle/Makefile:

* ``_build/liboracle.so`` — the CPU restatement (vq3r_oracle.c), built from
  this repository's sources; it exists on every machine the tests run on.
* ``_ref/libwaste_ref.so`` — the reference engine compiled from its own
  sources plus ref_harness.c; built only where the reference tree is
  present, and carried to GPU machines with the working copy.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
module; the product (warp_b200, libwaste_cuda.so) never imports it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libwaste_ref.so")


def reference_tree() -> str | None:
    """The sqliteai/warp source tree the checker is built from: the
    WARP_REFERENCE environment variable, else a checkout named `reference`
    beside this repository. None when neither holds a `src/` directory
    (machines that only run the prebuilt oracle/_ref)."""
    cand = os.environ.get("WARP_REFERENCE") or os.path.join(
        os.path.dirname(os.path.dirname(HERE)), "reference")
    return cand if os.path.isdir(os.path.join(cand, "src")) else None


REF_TREE = reference_tree()

P = C.c_void_p


def build(ref: bool | None = None):
    """make -C oracle (and `ref` when the reference tree is present)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    if ref is None:
        ref = REF_TREE is not None
    if ref:
        if REF_TREE is None:
            raise FileNotFoundError("the reference tree is not present: set WARP_REFERENCE")
        subprocess.run(["make", "-s", "-j8", "-C", HERE, "ref", f"REF={REF_TREE}"], check=True)


class OrcMoe(C.Structure):
    """orc_moe (vq3r_oracle.h)."""
    _fields_ = [("hidden", C.c_int), ("inter", C.c_int), ("n_experts", C.c_int),
                ("top_k", C.c_int), ("renorm", C.c_int), ("routed_scale", C.c_float),
                ("stages", C.c_int), ("entries", C.c_int), ("vec_dim", C.c_int),
                ("index_block", C.c_int), ("router", P), ("bias", P), ("books", P),
                ("n_books", C.c_int), ("bank", P), ("rec_bytes", C.c_size_t),
                ("shared_inter", C.c_int), ("sh_gate", P), ("sh_up", P), ("sh_down", P),
                ("sh_gate_s", P), ("sh_up_s", P), ("sh_down_s", P), ("sh_bits", C.c_int),
                ("sh_group", C.c_int), ("act_situ", C.c_int), ("situ_beta", C.c_float),
                ("situ_lbeta", C.c_float), ("index_bits", C.c_int)]


_orc = None
_ref = None


def _p(a):
    return C.c_void_p(a.ctypes.data) if a is not None else None


def lib() -> C.CDLL:
    global _orc
    if _orc is None:
        if not os.path.exists(ORACLE_SO):
            build(ref=False)
        L = C.CDLL(ORACLE_SO)
        L.orc_f16_flush.restype = C.c_float
        L.orc_f16_flush.argtypes = [C.c_uint16]
        L.orc_f16.restype = C.c_float
        L.orc_f16.argtypes = [C.c_uint16]
        L.orc_lut_build.argtypes = [P, P, C.c_int, P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]
        L.orc_vq_rows.argtypes = [P, P, P, P, C.c_int, C.c_int, C.c_int, C.c_int]
        L.orc_vq_matvec.argtypes = [P, P, P, P, C.c_int, C.c_int, P, C.c_int, C.c_int, C.c_int,
                                    C.c_int, P, C.c_int]
        L.orc_dequant.argtypes = [P, P, P, C.c_int, C.c_int, P, C.c_int, C.c_int, C.c_int,
                                  C.c_int, C.c_int]
        L.orc_vq4p_quant.argtypes = [P, C.c_int, P, P]
        L.orc_vq4p_rows.argtypes = [P, P, P, P, P, C.c_int, C.c_int]
        L.orc_vq4p_matvec.argtypes = [P, P, P, P, C.c_int, C.c_int, P, C.c_int, P, P, P,
                                      C.c_int]
        L.orc_set_exact_math.argtypes = [C.c_int]
        L.orc_vq_encode.argtypes = [P, C.c_int, P, C.c_int, C.c_int, C.c_int, P]
        L.orc_vq_lloyd.restype = C.c_int
        L.orc_vq_lloyd.argtypes = [P, C.c_int, P, C.c_int, C.c_int]
        L.orc_kda_step.argtypes = [C.c_int, C.c_int, C.c_int, P, P, P, P, P, P, P, P]
        L.orc_short_conv_step.argtypes = [C.c_int, C.c_int, P, P, P, P, P]
        L.orc_rmsnorm_gated.argtypes = [C.c_int, P, P, P, C.c_float, P]
        L.orc_dotf.restype = C.c_float
        L.orc_dotf.argtypes = [P, P, C.c_int]
        L.orc_route.argtypes = [P, P, C.c_int, C.c_int, C.c_int, C.c_float, P, P]
        L.orc_mvq_rows.argtypes = [P, P, P, P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_size_t]
        L.orc_record_check.argtypes = [C.POINTER(OrcMoe), C.c_int, C.c_int]
        L.orc_moe_layer.argtypes = [C.POINTER(OrcMoe), C.c_int, P, P, P, P, C.c_int]
        L.orc_rmsnorm.argtypes = [P, P, P, C.c_int, C.c_float]
        L.orc_situ_pair.restype = C.c_float
        L.orc_situ_pair.argtypes = [C.c_float, C.c_float, C.c_float, C.c_float]
        L.orc_moe_block.argtypes = [C.POINTER(OrcMoe), C.c_int, P, P, C.c_float, P, P, P,
                                    C.c_int]
        L.orc_moe_experts.argtypes = [C.POINTER(OrcMoe), P, P, C.c_int, P, P, C.c_int]
        L.orc_moe_chunk.argtypes = [C.POINTER(OrcMoe), C.c_int, P, C.c_int, P, P, P, C.c_int]
        _orc = L
    return _orc


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref() -> C.CDLL | None:
    global _ref
    if _ref is None:
        if not os.path.exists(REF_SO):
            return None
        _ref = _bind_refh(C.CDLL(REF_SO))
    return _ref


ENGINE_CUDA_SO = os.path.join(os.path.dirname(HERE), "integration", "_build",
                              "libwaste_engine_cuda.so")
_engine_cuda = None


def engine_cuda() -> C.CDLL | None:
    """The reference engine patched with the CUDA backend (integration/),
    with the same harness entry points as ref() plus refh_backend_auto and
    refh_moe_upload. Loads libwaste_cuda.so as its dependency (the same
    instance warp_b200 binds)."""
    global _engine_cuda
    if _engine_cuda is None:
        if not os.path.exists(ENGINE_CUDA_SO):
            return None
        R = _bind_refh(C.CDLL(ENGINE_CUDA_SO))
        R.refh_backend_auto.restype = C.c_char_p
        R.refh_moe_upload.restype = C.c_int
        R.refh_moe_upload.argtypes = [P]
        _engine_cuda = R
    return _engine_cuda


def _bind_refh(R: C.CDLL) -> C.CDLL:
    """ctypes signatures of the harness (ref_harness.c) and of the engine
    functions the checker calls."""
    R.refh_set_backend.restype = C.c_char_p
    R.refh_set_backend.argtypes = [C.c_int]
    R.refh_best_backend.restype = C.c_int
    R.refh_pool_init.argtypes = [C.c_int]
    R.refh_pool_threads.restype = C.c_int
    R.refh_version.restype = C.c_char_p
    R.refh_lutb.argtypes = [P, P, C.c_int, C.c_int, P, C.c_int, C.c_int, C.c_int, C.c_int]
    R.refh_vq_matvec.argtypes = [P, P, P, P, C.c_int, C.c_int, P, C.c_int, C.c_int,
                                 C.c_int, C.c_int, C.c_int]
    R.refh_mv_open.restype = P
    R.refh_mv_open.argtypes = [P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]
    R.refh_mv_run.argtypes = [P, P, P, P, P, C.c_int, C.c_int, C.c_int]
    R.refh_mv_close.argtypes = [P]
    R.refh_moe_open.restype = P
    R.refh_moe_open.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                C.c_float, P, P, P, C.c_int, C.c_int, P, C.c_size_t,
                                C.c_int, P, P, P, P, P, P, C.c_int, C.c_int]
    R.refh_vq4p_matvec.argtypes = [P, P, P, P, C.c_int, C.c_int, P, C.c_int, C.c_int]
    R.refh_vq4p_table.argtypes = [P, P, P, C.c_int, P, C.c_int, C.c_int]
    R.refh_moe_layer.restype = C.c_int
    R.refh_moe_layer.argtypes = [P, P, P, P]
    R.refh_moe_chunk.restype = C.c_int
    R.refh_moe_chunk.argtypes = [P, P, C.c_int, P, P, P]
    R.refh_moe_close.argtypes = [P]
    R.refh_load.restype = P
    R.refh_load.argtypes = [C.c_char_p]
    R.refh_codebooks.restype = C.POINTER(C.c_float)
    R.refh_codebooks.argtypes = [P, C.POINTER(C.c_int)]
    R.refh_free.argtypes = [P]
    R.waste_rmsnorm.argtypes = [P, P, P, C.c_int, C.c_float]
    R.waste_mvq_rows_f32.argtypes = [C.c_int, C.c_int, P]
    R.refh_moe_set_act.argtypes = [P, C.c_int, C.c_float, C.c_float]
    R.waste_vq_encode.argtypes = [P, C.c_int, P, C.c_int, C.c_int, C.c_int, P, C.c_int]
    R.waste_vq_lloyd.restype = C.c_int
    R.waste_vq_lloyd.argtypes = [P, C.c_int, P, C.c_int, C.c_int, C.c_int]
    R.waste_kda_step.argtypes = [C.c_int, C.c_int, C.c_int, P, P, P, P, P, P, P, P]
    R.waste_short_conv_step.argtypes = [C.c_int, C.c_int, P, P, P, P, P]
    R.waste_rmsnorm_gated.argtypes = [C.c_int, P, P, P, C.c_float, P]
    R.waste_situ_pair.restype = C.c_float
    R.waste_situ_pair.argtypes = [C.c_float, C.c_float, C.c_float, C.c_float]
    return R


# ---- restatement ----------------------------------------------------------

def f16_flush(raw: np.ndarray) -> np.ndarray:
    L = lib()
    r = np.asarray(raw, dtype=np.uint16).ravel()
    return np.array([L.orc_f16_flush(int(v)) for v in r], dtype=np.float32).reshape(np.shape(raw))


def lut_build(books, cb_base, x, stages=3, fma=1):
    b = np.ascontiguousarray(books, dtype=np.float32)
    xx = np.ascontiguousarray(x, dtype=np.float32)
    nv = xx.size // 8
    lut = np.empty((nv, stages, 256), dtype=np.float32)
    lib().orc_lut_build(_p(lut), _p(b), cb_base, _p(xx), nv, stages, 256, 8, fma)
    return lut


def vq_matvec(idx, scale, x, M, N, books, cb_base, stages=3, fma=1):
    i = np.ascontiguousarray(idx, dtype=np.uint8)
    s = np.ascontiguousarray(scale, dtype=np.uint16)
    xx = np.ascontiguousarray(x, dtype=np.float32)
    b = np.ascontiguousarray(books, dtype=np.float32)
    y = np.empty(M, dtype=np.float32)
    lut = np.empty((N // 8) * stages * 256, dtype=np.float32)
    lib().orc_vq_matvec(_p(y), _p(i), _p(s), _p(xx), M, N, _p(b), cb_base, stages, 256, 8,
                        _p(lut), fma)
    return y


def vq4p_matvec(idx, scale, x, M, N, books, cb_base, fma=1):
    """A VQ4P matrix (books [n][64][8], flushed) times x."""
    i = np.ascontiguousarray(idx, dtype=np.uint8)
    s = np.ascontiguousarray(scale, dtype=np.uint16)
    xx = np.ascontiguousarray(x, dtype=np.float32)
    b = np.ascontiguousarray(books, dtype=np.float32)
    nv = N // 8
    y = np.empty(M, dtype=np.float32)
    lut = np.empty(nv * 256, dtype=np.float32)
    q = np.empty(nv * 256, dtype=np.int8)
    qs = np.empty(nv // 32 + 2, dtype=np.float32)
    lib().orc_vq4p_matvec(_p(y), _p(i), _p(s), _p(xx), M, N, _p(b), cb_base, _p(lut), _p(q),
                          _p(qs), fma)
    return y


def lut_build_en(books, cb_base, x, stages, entries, fma=1):
    b = np.ascontiguousarray(books, dtype=np.float32)
    xx = np.ascontiguousarray(x, dtype=np.float32)
    nv = xx.size // 8
    lut = np.empty((nv, stages, entries), dtype=np.float32)
    lib().orc_lut_build(_p(lut), _p(b), cb_base, _p(xx), nv, stages, entries, 8, fma)
    return lut


def vq4p_table(books, cb_base, x, fma=1):
    """The int8 VQ4P tables of x: q [N/8][4][64], qs [ceil(N/256)]."""
    nv = np.size(x) // 8
    lut = lut_build_en(books, cb_base, x, 4, 64, fma)
    q = np.empty((nv, 4, 64), dtype=np.int8)
    qs = np.empty((nv + 31) // 32, dtype=np.float32)
    lib().orc_vq4p_quant(_p(lut), nv, _p(q), _p(qs))
    return q, qs


def ref_vq4p_matvec(idx, scale, x, M, N, books, cb_base):
    """The compiled reference's vq_matvec on a VQ4P matrix (LUT backend:
    the best this host has), through the harness."""
    R = ref()
    R.refh_set_backend(R.refh_best_backend())
    i = np.ascontiguousarray(idx, dtype=np.uint8)
    s = np.ascontiguousarray(scale, dtype=np.uint16)
    xx = np.ascontiguousarray(x, dtype=np.float32)
    b = np.ascontiguousarray(books, dtype=np.float32)
    y = np.empty(M, dtype=np.float32)
    R.refh_vq4p_matvec(_p(y), _p(i), _p(s), _p(xx), M, N, _p(b), b.shape[0], cb_base)
    return y


def ref_vq4p_table(books, cb_base, x):
    R = ref()
    R.refh_set_backend(R.refh_best_backend())
    xx = np.ascontiguousarray(x, dtype=np.float32)
    b = np.ascontiguousarray(books, dtype=np.float32)
    nv = xx.size // 8
    q = np.empty((nv, 4, 64), dtype=np.int8)
    qs = np.empty(nv // 32 + 2, dtype=np.float32)
    R.refh_vq4p_table(_p(q), _p(qs), _p(xx), xx.size, _p(b), b.shape[0], cb_base)
    return q, qs[: (nv + 31) // 32]


def dequant(idx, scale, M, N, books, cb_base, stages=3):
    i = np.ascontiguousarray(idx, dtype=np.uint8)
    s = np.ascontiguousarray(scale, dtype=np.uint16)
    b = np.ascontiguousarray(books, dtype=np.float32)
    W = np.empty((M, N), dtype=np.float32)
    lib().orc_dequant(_p(W), _p(i), _p(s), M, N, _p(b), cb_base, stages, 256, 8, 64)
    return W


def route(logits, bias, K, renorm, routed_scale):
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    b = np.ascontiguousarray(bias, dtype=np.float32) if bias is not None else None
    idx = np.empty(K, dtype=np.int32)
    w = np.empty(K, dtype=np.float32)
    lib().orc_route(_p(lg), _p(b), lg.size, K, renorm, C.c_float(routed_scale), _p(idx), _p(w))
    return idx, w


def _moe_struct(L, keep):
    books = np.ascontiguousarray(L.books)
    router = np.ascontiguousarray(L.router, dtype=np.float32)
    keep += [books, router, L.bank]
    s = OrcMoe()
    s.hidden, s.inter, s.n_experts, s.top_k = L.hidden, L.inter, L.n_experts, L.top_k
    s.renorm, s.routed_scale = L.renorm, L.routed_scale
    p6 = L.stages == 4               # VQ4P: four stages of 64, packed indices
    s.stages, s.entries, s.vec_dim, s.index_block = L.stages, 64 if p6 else 256, 8, 64
    s.index_bits = 6 if p6 else 8
    s.router, s.books, s.n_books = _p(router), _p(books), books.shape[0]
    if L.bias is not None:
        b = np.ascontiguousarray(L.bias, dtype=np.float32)
        keep.append(b)
        s.bias = _p(b)
    s.bank, s.rec_bytes = _p(L.bank), L.rec_bytes
    s.shared_inter = L.shared_inter
    if L.shared_inter:
        for k in ("gate", "up", "down"):
            q, sc = L.sh[k]
            keep += [q, sc]
            setattr(s, "sh_" + k, _p(q))
            setattr(s, "sh_" + k + "_s", _p(sc))
        s.sh_bits, s.sh_group = 8, 128
    s.act_situ = int(getattr(L, "act_situ", 0))
    s.situ_beta = float(getattr(L, "situ_beta", 0.0))
    s.situ_lbeta = float(getattr(L, "situ_lbeta", 0.0))
    return s


def moe_layer(L, x, fma=1):
    keep = []
    s = _moe_struct(L, keep)
    xx = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(L.hidden, dtype=np.float32)
    idx = np.empty(L.top_k, dtype=np.int32)
    w = np.empty(L.top_k, dtype=np.float32)
    rc = lib().orc_moe_layer(C.byref(s), L.layer, _p(xx), _p(out), _p(idx), _p(w), fma)
    if rc:
        raise RuntimeError("oracle: record check failed")
    return out, idx, w


def situ_pair(g, u, beta, lbeta):
    """src/model.c:505-509, per element (restatement)."""
    gg = np.ascontiguousarray(g, dtype=np.float32).ravel()
    uu = np.ascontiguousarray(u, dtype=np.float32).ravel()
    f = lib().orc_situ_pair
    return np.array([f(C.c_float(a), C.c_float(b), C.c_float(beta), C.c_float(lbeta))
                     for a, b in zip(gg, uu)], dtype=np.float32).reshape(np.shape(g))


def mvq_rows(raw, scales, x, inp, group, bits, rowbytes):
    """src/model.c:265-320 waste_mvq_rows_f32 (restatement): y[rows]."""
    r = np.ascontiguousarray(raw, dtype=np.uint8)
    s = np.ascontiguousarray(scales, dtype=np.uint16)
    xx = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(r.shape[0], dtype=np.float32)
    lib().orc_mvq_rows(_p(y), _p(r), _p(s), _p(xx), r.shape[0], inp, group, bits, rowbytes)
    return y


class MvqArg(C.Structure):
    """mvq_arg (src/simd.h:35-39): the engine's argument of mvq_rows_f32."""
    _fields_ = [("y", P), ("W", P), ("ws", P), ("xq", P), ("xs", P), ("in_", C.c_int),
                ("ng", C.c_int), ("group", C.c_int), ("bits", C.c_int), ("rowbytes", C.c_size_t)]


def ref_mvq_rows(raw, scales, x, inp, group, bits, rowbytes):
    """The reference's own portable waste_mvq_rows_f32, compiled."""
    R = ref()
    if R is None:
        raise RuntimeError("oracle/_ref/libwaste_ref.so is not built")
    r = np.ascontiguousarray(raw, dtype=np.uint8)
    s = np.ascontiguousarray(scales, dtype=np.uint16)
    xx = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(r.shape[0], dtype=np.float32)
    a = MvqArg(_p(y), _p(r), _p(s), None, _p(xx), inp, (inp + group - 1) // group, group, bits,
               rowbytes)
    R.waste_mvq_rows_f32(0, r.shape[0], C.byref(a))
    return y


def rmsnorm(x, w, eps):
    """src/model.c:132-138 (serial fp32 sum of squares)."""
    xx = np.ascontiguousarray(x, dtype=np.float32)
    ww = np.ascontiguousarray(w, dtype=np.float32)
    o = np.empty_like(xx)
    lib().orc_rmsnorm(_p(o), _p(xx), _p(ww), xx.size, C.c_float(eps))
    return o


def moe_block(L, h, norm_w, eps, fma=1):
    """h + moe_layer(rmsnorm(h)): (h_out, idx, w)."""
    keep = []
    s = _moe_struct(L, keep)
    hh = np.ascontiguousarray(h, dtype=np.float32)
    nw = np.ascontiguousarray(norm_w, dtype=np.float32)
    out = np.empty(L.hidden, dtype=np.float32)
    idx = np.empty(L.top_k, dtype=np.int32)
    w = np.empty(L.top_k, dtype=np.float32)
    rc = lib().orc_moe_block(C.byref(s), L.layer, _p(hh), _p(nw), C.c_float(eps), _p(out),
                             _p(idx), _p(w), fma)
    if rc:
        raise RuntimeError("oracle: record check failed")
    return out, idx, w


def moe_experts(L, idx, w, x, fma=1):
    keep = []
    s = _moe_struct(L, keep)
    i = np.ascontiguousarray(idx, dtype=np.int32)
    ww = np.ascontiguousarray(w, dtype=np.float32)
    xx = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(L.hidden, dtype=np.float32)
    lib().orc_moe_experts(C.byref(s), _p(i), _p(ww), i.size, _p(xx), _p(y), fma)
    return y


def moe_chunk(L, x, fma=1):
    keep = []
    s = _moe_struct(L, keep)
    xx = np.ascontiguousarray(x, dtype=np.float32)
    nT = xx.shape[0]
    out = np.empty((nT, L.hidden), dtype=np.float32)
    route_ = np.empty((nT, L.top_k), dtype=np.int32)
    rw = np.empty((nT, L.top_k), dtype=np.float32)
    rc = lib().orc_moe_chunk(C.byref(s), L.layer, _p(xx), nT, _p(out), _p(route_), _p(rw), fma)
    if rc:
        raise RuntimeError("oracle: record check failed")
    return out, route_, rw


# ---- the reference, compiled ---------------------------------------------

def ref_rmsnorm(x, w, eps):
    """The reference's own waste_rmsnorm (src/model.c:132-138), compiled."""
    R = ref()
    if R is None:
        raise RuntimeError("oracle/_ref/libwaste_ref.so is not built")
    xx = np.ascontiguousarray(x, dtype=np.float32)
    ww = np.ascontiguousarray(w, dtype=np.float32)
    o = np.empty_like(xx)
    R.waste_rmsnorm(_p(o), _p(xx), _p(ww), xx.size, C.c_float(eps))
    return o


def ref_situ_pair(g, u, beta, lbeta):
    """The reference's own waste_situ_pair (src/model.c:505-509), per element."""
    R = ref()
    if R is None:
        raise RuntimeError("oracle/_ref/libwaste_ref.so is not built")
    gg = np.ascontiguousarray(g, dtype=np.float32).ravel()
    uu = np.ascontiguousarray(u, dtype=np.float32).ravel()
    return np.array([R.waste_situ_pair(C.c_float(a), C.c_float(b), C.c_float(beta),
                                       C.c_float(lbeta)) for a, b in zip(gg, uu)],
                    dtype=np.float32).reshape(np.shape(g))


class RefMoe:
    """One MoE layer inside the reference engine (ref_harness.c)."""

    def __init__(self, L, max_tokens=64, backend=None, threads=0, lib=None):
        R = lib if lib is not None else ref()
        if R is None:
            raise RuntimeError("oracle/_ref/libwaste_ref.so is not built")
        self.R = R
        self.backend = R.refh_set_backend(R.refh_best_backend() if backend is None else backend)
        R.refh_pool_init(threads)
        self.keep = [np.ascontiguousarray(L.router, dtype=np.float32),
                     np.ascontiguousarray(L.books, dtype=np.float32), L.bank]
        bias = np.ascontiguousarray(L.bias, dtype=np.float32) if L.bias is not None else None
        self.keep.append(bias)
        sh = [None] * 6
        if L.shared_inter:
            sh = []
            for k in ("gate", "up", "down"):
                q, s = L.sh[k]
                self.keep += [q, s]
                sh += [_p(q), _p(s)]
        self.h = R.refh_moe_open(L.layer, L.hidden, L.inter, L.n_experts, L.top_k, L.renorm,
                                 C.c_float(L.routed_scale), _p(self.keep[0]), _p(bias),
                                 _p(self.keep[1]), self.keep[1].shape[0], L.cb_base,
                                 _p(L.bank), L.rec_bytes, L.shared_inter, *sh, max_tokens,
                                 6 if L.stages == 4 else 8)
        if not self.h:
            raise RuntimeError("reference harness refused the layer "
                               "(the shared width must be a multiple of inter)")
        if getattr(L, "act_situ", 0):
            R.refh_moe_set_act(self.h, 1, C.c_float(L.situ_beta), C.c_float(L.situ_lbeta))
        self.L = L

    def layer(self, x):
        xx = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty(self.L.hidden, dtype=np.float32)
        idx = np.empty(self.L.top_k, dtype=np.int32)
        rc = self.R.refh_moe_layer(self.h, _p(xx), _p(out), _p(idx))
        if rc:
            raise RuntimeError(f"reference read error {rc}")
        return out, idx

    def chunk(self, x):
        xx = np.ascontiguousarray(x, dtype=np.float32)
        nT = xx.shape[0]
        out = np.empty((nT, self.L.hidden), dtype=np.float32)
        r = np.empty((nT, self.L.top_k), dtype=np.int32)
        w = np.empty((nT, self.L.top_k), dtype=np.float32)
        rc = self.R.refh_moe_chunk(self.h, _p(xx), nT, _p(out), _p(r), _p(w))
        if rc:
            raise RuntimeError(f"reference read error {rc}")
        return out, r, w

    def close(self):
        if self.h:
            self.R.refh_moe_close(self.h)
            self.h = None


class exact_math:
    """Within this context the restatement's activation (and KDA) exp/tanh
    are correctly rounded (the device's arithmetic where it rounds them
    correctly) rather than libm's: `with O.exact_math(): ...`."""

    def __enter__(self):
        lib().orc_set_exact_math(1)
        return self

    def __exit__(self, *exc):
        lib().orc_set_exact_math(0)
        return False


# ---- KDA (src/kda.c) --------------------------------------------------------

def _kda(fn, H, K, V, q, k, v, g, beta, S):
    a = [np.ascontiguousarray(t, dtype=np.float32) for t in (q, k, v, g, beta)]
    S2 = np.array(S, dtype=np.float32, copy=True, order="C")
    o = np.empty(H * V, dtype=np.float32)
    u = np.empty(V, dtype=np.float32)
    fn(H, K, V, *[_p(t) for t in a], _p(S2), _p(o), _p(u))
    return S2, o


def kda_step(H, K, V, q, k, v, g, beta, S):
    """One KDA decode step: returns (new state, o); S is not modified."""
    return _kda(lib().orc_kda_step, H, K, V, q, k, v, g, beta, S)


def ref_kda_step(H, K, V, q, k, v, g, beta, S):
    """The compiled reference's waste_kda_step (src/kda.c:26-68)."""
    return _kda(ref().waste_kda_step, H, K, V, q, k, v, g, beta, S)


def _conv(fn, C_, KS, w, bias, ring, x):
    ww = np.ascontiguousarray(w, dtype=np.float32)
    bb = np.ascontiguousarray(bias, dtype=np.float32) if bias is not None else None
    r2 = np.array(ring, dtype=np.float32, copy=True, order="C")
    xx = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(C_, dtype=np.float32)
    fn(C_, KS, _p(ww), _p(bb), _p(r2), _p(xx), _p(y))
    return r2, y


def short_conv_step(C_, KS, w, bias, ring, x):
    """Returns (new ring, y); ring is not modified."""
    return _conv(lib().orc_short_conv_step, C_, KS, w, bias, ring, x)


def ref_short_conv_step(C_, KS, w, bias, ring, x):
    return _conv(ref().waste_short_conv_step, C_, KS, w, bias, ring, x)


def _rg(fn, C_, x, gate, w, eps):
    a = [np.ascontiguousarray(t, dtype=np.float32) for t in (x, gate, w)]
    y = np.empty(C_, dtype=np.float32)
    fn(C_, _p(a[0]), _p(a[1]), _p(a[2]), C.c_float(eps), _p(y))
    return y


def rmsnorm_gated(C_, x, gate, w, eps):
    return _rg(lib().orc_rmsnorm_gated, C_, x, gate, w, eps)


def ref_rmsnorm_gated(C_, x, gate, w, eps):
    return _rg(ref().waste_rmsnorm_gated, C_, x, gate, w, eps)


# ---- the converter's RVQ encoder (src/vq.c) --------------------------------------

def vq_encode(X, books):
    """X [n][dim], books [stages][entries][dim] -> codes [n][stages]."""
    xx = np.ascontiguousarray(X, dtype=np.float32)
    bb = np.ascontiguousarray(books, dtype=np.float32)
    out = np.empty((xx.shape[0], bb.shape[0]), dtype=np.uint8)
    lib().orc_vq_encode(_p(xx), xx.shape[0], _p(bb), bb.shape[0], bb.shape[1], xx.shape[1],
                        _p(out))
    return out


def ref_vq_encode(X, books, threads=0):
    """The compiled reference's waste_vq_encode (its thread pool)."""
    xx = np.ascontiguousarray(X, dtype=np.float32)
    bb = np.ascontiguousarray(books, dtype=np.float32)
    out = np.empty((xx.shape[0], bb.shape[0]), dtype=np.uint8)
    ref().waste_vq_encode(_p(xx), xx.shape[0], _p(bb), bb.shape[0], bb.shape[1], xx.shape[1],
                          _p(out), threads)
    return out


def vq_lloyd(X, C):
    """(new centroids, non-empty clusters)."""
    xx = np.ascontiguousarray(X, dtype=np.float32)
    cc = np.array(C, dtype=np.float32, copy=True, order="C")
    live = lib().orc_vq_lloyd(_p(xx), xx.shape[0], _p(cc), cc.shape[0], cc.shape[1])
    return cc, live


def ref_vq_lloyd(X, C, threads=0):
    xx = np.ascontiguousarray(X, dtype=np.float32)
    cc = np.array(C, dtype=np.float32, copy=True, order="C")
    live = ref().waste_vq_lloyd(_p(xx), xx.shape[0], _p(cc), cc.shape[0], cc.shape[1], threads)
    return cc, live
