"""Regenerates the golden fixtures in tests/golden/ from the REFERENCE.

Run on a machine that has the reference tree (WARP_REFERENCE, or a checkout
named `reference` beside this repository) and
oracle/_ref/libwaste_ref.so built from it (make -C oracle ref):

    python tests/golden/make_golden.py

Every output here is produced by the reference's own code:

* f16_flush.npz — all 65536 f16 bit patterns through the engine's codebook
  decode (src/model.c:1278-1287), reached by loading a container whose
  codebooks.bin holds every pattern. The container is written by the
  reference's tools/make_test_container.py (imported from the reference
  tree, seed 0), and its codebooks.bin is then replaced.
* lut_*.npz, matvec_*.npz — vq_build_lut / vq_matvec (src/model.c:1911,
  2282) through the reference's AVX-512 slot and its portable (CPU) slot.
* vq4p.npz, moe_vq4p*.npz — the VQ4P format (src/model.c:2026-2229): the
  matvec, its int8 tables, and VQ4P MoE layers.
* kda.npz — the KDA kernels (src/kda.c:26-111) on seeded inputs.
* enc.npz — the converter's encoder and Lloyd step (src/vq.c:50-136).
* moe_*.npz — moe_layer / moe_chunk (src/model.c:2713, 3512) on seeded
  layers built by warp_b200.synth; the inputs are regenerated from the seed
  (numpy PCG64, which is stable across numpy versions) and pinned by a
  sha256 of their bytes.

The fixtures are small; tests compare the CPU restatement against them
bit for bit and the CUDA backend within the stated tolerances.
"""
from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import struct
import sys
import tempfile
import zlib

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import oracle as O  # noqa: E402
from warp_b200 import synth  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))
REF_TREE = O.REF_TREE
if REF_TREE is None:
    raise SystemExit("make_golden.py needs the reference tree: set WARP_REFERENCE")

sys.path.insert(0, os.path.join(ROOT, "tests"))
from golden_cases import (CONV_C, CONV_KS, KDA_CASES, MOE_CASES, MVQ_CASES,  # noqa: E402
                          NORM_DIM, NORM_HEADS, NORM_SIZES, VQ4P_CASES, VQ4P_MOE_CASES,
                          conv_inputs, kda_inputs, norm_inputs, sha, vq4p_books,
                          vq4p_case, ENC_CASES, LLOYD_CASES, enc_inputs,
                          lloyd_inputs)  # shared with the tests


def layer_sha(L) -> str:
    h = hashlib.sha256()
    for a in (L.books_raw, L.router, L.bank):
        h.update(np.ascontiguousarray(a).tobytes())
    if L.bias is not None:
        h.update(L.bias.tobytes())
    for k in ("gate", "up", "down"):
        if k in L.sh:
            h.update(L.sh[k][0].tobytes())
            h.update(L.sh[k][1].tobytes())
    return h.hexdigest()


def f16_flush_fixture(R):
    sys.path.insert(0, os.path.join(REF_TREE, "tools"))
    import make_test_container as mtc  # the reference's own generator
    tmp = tempfile.mkdtemp(prefix="golden_ct_")
    try:
        argv = sys.argv
        sys.argv = ["make_test_container.py", tmp, "--seed", "0"]
        try:
            mtc.main()
        finally:
            sys.argv = argv
        allpat = np.arange(65536, dtype=np.uint32).astype(np.uint16)
        n_books = 65536 // (256 * 8)
        with open(os.path.join(tmp, "codebooks.bin"), "wb") as f:
            for b in range(n_books):
                f.write(struct.pack("<IHBBII", 0x4B424357, b, 4, 8, 256, 0))
                f.write(allpat[b * 2048:(b + 1) * 2048].tobytes())
        m = R.refh_load(tmp.encode())
        if not m:
            raise RuntimeError("reference could not load the container")
        n = O.C.c_int(0)
        p = R.refh_codebooks(m, O.C.byref(n))
        got = np.ctypeslib.as_array(p, shape=(n.value * 2048,)).copy()
        R.refh_free(m)
        np.savez_compressed(os.path.join(OUT, "f16_flush.npz"),
                            bits=got.view(np.uint32))
        print("f16_flush.npz", n.value, "books")
    finally:
        shutil.rmtree(tmp, ignore_errors=True)


def lut_matvec_fixtures(R):
    rng = np.random.default_rng(2024)
    raw = synth.codebooks(rng, 12)
    books = synth.flush_f16(raw)
    cases = {"matvec_ragged": (100, 256, 3), "matvec_square": (256, 512, 3),
             "matvec_vq2r": (192, 128, 2)}
    xs = {}
    for be, tag in ((1, "avx512"), (0, "cpu")):
        name = R.refh_set_backend(be)
        x = synth.activations(99, 512)[0]
        lut = np.empty((64, 3, 256), np.float32)
        R.refh_lutb(O._p(lut), O._p(books), 12, 3, O._p(x), 64, 3, 256, 8)
        np.savez_compressed(os.path.join(OUT, f"lut_{tag}.npz"), books_raw=raw, x=x,
                            cb_base=3, lut=lut, backend=name)
        for cname, (M, N, st) in cases.items():
            r2 = np.random.default_rng(zlib.crc32(cname.encode()))
            idx, sc = synth.random_matrix(r2, M, N, stages=st)
            if cname not in xs:
                xs[cname] = synth.activations(len(cname), N)[0]
            x = xs[cname]
            y = np.empty(M, np.float32)
            R.refh_vq_matvec(O._p(y), O._p(idx), O._p(sc), O._p(x), M, N, O._p(books), 12,
                             3, st, 256, 8)
            np.savez_compressed(os.path.join(OUT, f"{cname}_{tag}.npz"), books_raw=raw,
                                idx=idx, scale=sc, x=x, y=y, M=M, N=N, stages=st,
                                cb_base=3, backend=name)
        print("lut/matvec fixtures for", name)


def moe_fixtures(only=None, cases=MOE_CASES):
    for name, (seed, kw, xseed, T) in cases.items():
        if only and name not in only:
            continue
        L = synth.moe_layer(seed, **kw)
        x = synth.activations(xseed, L.hidden, T=max(T, 2))
        res = {"sha": layer_sha(L), "seed": seed, "xseed": xseed}
        for be, tag in ((1, "avx512"), (0, "cpu")):
            rm = O.RefMoe(L, max_tokens=max(T, 1), backend=be, threads=0)
            out0, idx0 = rm.layer(x[0])
            out1, idx1 = rm.layer(x[1])
            res[f"out0_{tag}"], res[f"idx0_{tag}"] = out0, idx0
            res[f"out1_{tag}"], res[f"idx1_{tag}"] = out1, idx1
            if T:
                c, r, w = rm.chunk(x[:T])
                res[f"chunk_{tag}"], res[f"route_{tag}"], res[f"rw_{tag}"] = c, r, w
            res[f"backend_{tag}"] = rm.backend
            rm.close()
        np.savez_compressed(os.path.join(OUT, f"{name}.npz"), **res)
        print(name, "written")


def vq4p_fixtures():
    """VQ4P (src/model.c:2026-2229): vq_matvec and vq_build_lut's int8
    shadow through the reference with its best LUT backend (AVX-512 here),
    on seeded packed matrices (regenerated by golden_cases.vq4p_case and
    pinned by a sha256); then moe_layer / moe_chunk on VQ4P layers."""
    raw = vq4p_books()
    books = synth.flush_f16(raw)
    res = {"books_sha": sha(raw), "cb_base": np.int64(4)}
    for name in VQ4P_CASES:
        idx, sc, x, M, N = vq4p_case(name)
        res[f"{name}_sha"] = sha(idx, sc, x)
        res[f"{name}_y"] = O.ref_vq4p_matvec(idx, sc, x, M, N, books, 4)
        q, qs = O.ref_vq4p_table(books, 4, x)
        res[f"{name}_q"], res[f"{name}_qs"] = q, qs
    R = O.ref()
    res["backend"] = R.refh_set_backend(R.refh_best_backend())
    np.savez_compressed(os.path.join(OUT, "vq4p.npz"), **res)
    print("vq4p.npz written")
    moe_fixtures(cases=VQ4P_MOE_CASES)


def kda_fixture():
    """The reference's KDA kernels (src/kda.c:26-111: waste_kda_step,
    waste_short_conv_step, waste_rmsnorm_gated) on seeded inputs: the state
    (by a sha256) and output after every step of each case, three conv steps
    from a zero ring, and the gated norm of every head."""
    res = {}
    for name, (H, K, V, T) in KDA_CASES.items():
        S = np.zeros((H, K, V), np.float32)
        for t, (q, k, v, g, beta) in enumerate(kda_inputs(name)):
            S, o = O.ref_kda_step(H, K, V, q, k, v, g, beta, S)
            res[f"{name}_o{t}"] = o
        res[f"{name}_S_sha"] = sha(S)      # the final state, pinned by its bytes
    w, xs = conv_inputs()
    ring = np.zeros((CONV_C, CONV_KS - 1), np.float32)
    for t in range(xs.shape[0]):
        ring, y = O.ref_short_conv_step(CONV_C, CONV_KS, w, None, ring, xs[t])
        res[f"conv_y{t}"] = y
    res["conv_ring"] = ring
    x, gate, wn, eps = norm_inputs()
    res["norm_y"] = np.concatenate([
        O.ref_rmsnorm_gated(NORM_DIM, x[h * NORM_DIM:(h + 1) * NORM_DIM],
                            gate[h * NORM_DIM:(h + 1) * NORM_DIM], wn, float(eps))
        for h in range(NORM_HEADS)])
    np.savez_compressed(os.path.join(OUT, "kda.npz"), **res)
    print("kda.npz written")


def enc_fixture():
    """The reference's waste_vq_encode and waste_vq_lloyd (src/vq.c:50-136)
    on seeded inputs (regenerated by golden_cases and pinned by a sha256):
    the codes of every encoder case, and the centroids and live count after
    one Lloyd iteration."""
    res = {}
    for name in ENC_CASES:
        X, books = enc_inputs(name)
        res[f"{name}_sha"] = sha(X, books)
        res[f"{name}_codes"] = O.ref_vq_encode(X, books)
    for name in LLOYD_CASES:
        X, C0 = lloyd_inputs(name)
        res[f"{name}_sha"] = sha(X, C0)
        res[f"{name}_C"], res[f"{name}_live"] = O.ref_vq_lloyd(X, C0)
    np.savez_compressed(os.path.join(OUT, "enc.npz"), **res)
    print("enc.npz written")


def tiny_container():
    """tests/golden/tiny_container/: the reference's own test container
    (tools/make_test_container.py, seed 0: a Kimi-Linear at 1/18 scale, 4
    layers, 8 VQ3R experts top-2, 0.8 MB), for driving the engine through
    its public API with and without the CUDA backend."""
    out = os.path.join(OUT, "tiny_container")
    shutil.rmtree(out, ignore_errors=True)
    subprocess.run([sys.executable, os.path.join(REF_TREE, "tools", "make_test_container.py"),
                    out, "--seed", "0"], check=True)
    print("tiny_container written")


def mvq_fixture():
    """The reference's waste_mvq_rows_f32 (src/model.c:265-320, the trunk
    matvec the mvq_rows_f32 slot replaces) on seeded Q8G/Q4G/Q3G tensors."""
    res = {}
    for name, (rows, inp, bits) in MVQ_CASES.items():
        rng = np.random.default_rng(zlib.crc32(name.encode()))
        raw, s, rb = synth.trunk_tensor(rng, rows, inp, bits)
        x = synth.activations(len(name) + rows, inp)[0]
        res[f"{name}_raw"], res[f"{name}_s"], res[f"{name}_x"] = raw, s, x
        res[f"{name}_rowbytes"] = np.int64(rb)
        res[f"{name}_y"] = O.ref_mvq_rows(raw, s, x, inp, 128, bits, rb)
    np.savez_compressed(os.path.join(OUT, "mvq.npz"), **res)
    print("mvq.npz written")


def norm_fixture():
    """The reference's waste_rmsnorm (src/model.c:132-138) on seeded inputs:
    the rmsnorm in front of every MoE block of a decode step."""
    res = {}
    for n in NORM_SIZES:
        x = synth.activations(7000 + n, n)[0] * np.float32(3.0)
        w = synth.norm_weight(7100 + n, n)
        res[f"x{n}"], res[f"w{n}"] = x, w
        res[f"out{n}"] = O.ref_rmsnorm(x, w, synth.NORM_EPS)
    res["eps"] = np.float32(synth.NORM_EPS)
    np.savez_compressed(os.path.join(OUT, "norm.npz"), **res)
    print("norm.npz written")


def main():
    R = O.ref()
    if R is None:
        raise SystemExit("build the reference first: make -C oracle ref")
    f16_flush_fixture(R)
    lut_matvec_fixtures(R)
    moe_fixtures()
    norm_fixture()
    tiny_container()
    mvq_fixture()
    vq4p_fixtures()
    kda_fixture()
    enc_fixture()


if __name__ == "__main__":
    if sys.argv[1:] == ["norm"]:
        norm_fixture()
    elif sys.argv[1:2] == ["moe"]:
        moe_fixtures(sys.argv[2:])
    elif sys.argv[1:] == ["container"]:
        tiny_container()
    elif sys.argv[1:] == ["mvq"]:
        mvq_fixture()
    elif sys.argv[1:] == ["vq4p"]:
        vq4p_fixtures()
    elif sys.argv[1:] == ["kda"]:
        kda_fixture()
    elif sys.argv[1:] == ["enc"]:
        enc_fixture()
    else:
        main()
