"""The synthetic generator writes the reference's formats."""
import os
import sys

import numpy as np
import pytest

import oracle as O
from warp_b200 import synth

REF_TOOLS = os.path.join(O.REF_TREE, "tools") if O.REF_TREE else ""


def test_block_roundtrip():
    rng = np.random.default_rng(0)
    for M, N, st in ((100, 64, 3), (64, 8, 2), (1, 256, 3), (130, 40, 3)):
        idx = rng.integers(0, 256, size=(M, N // 8, st), dtype=np.uint8)
        b = synth.block_indices(idx)
        assert b.size == synth.index_bytes(M, N, st)
        assert np.array_equal(synth.unblock_indices(b, M, N, st), idx)
        # padding rows are zero
        nb = (M + 63) // 64
        full = b.reshape(nb, N // 8, 64, st)
        assert not full[-1, :, M - (nb - 1) * 64:, :].any()


@pytest.mark.skipif(not os.path.isdir(REF_TOOLS), reason="reference tree not present")
def test_block_layout_matches_reference_tool():
    sys.path.insert(0, REF_TOOLS)
    import make_test_container as mtc
    rng = np.random.default_rng(1)
    M, N = 70, 24
    idx = rng.integers(0, 256, size=(M, N // 8, 3), dtype=np.uint8)
    ref_layout = mtc.block_indices([list(idx[:, :, s].reshape(-1)) for s in range(3)], M, N)
    assert synth.block_indices(idx).tobytes() == ref_layout


def test_record_header_and_check():
    L = synth.moe_layer(3, hidden=128, inter=64, n_experts=4, top_k=2, shared_inter=0)
    for e in range(4):
        h = synth.parse_header(L.record(e))
        assert h["magic"] == synth.MAGIC_EXPERT and h["expert_id"] == e
        assert h["gate_off"] == 48 and h["rec_4k_blocks"] * 4096 == L.rec_bytes
        assert (h["up_off"] - h["gate_off"]) == synth.index_bytes(64, 128, 3)
    keep = []
    s = O._moe_struct(L, keep)
    for e in range(4):
        assert O.lib().orc_record_check(O.C.byref(s), L.layer, e) == 0
    # the wrong identity is refused, as record_check refuses it
    assert O.lib().orc_record_check(O.C.byref(s), L.layer + 1, 0) == -1


def test_record_crc_is_zlib():
    import zlib
    L = synth.moe_layer(4, hidden=64, inter=64, n_experts=1, top_k=1, shared_inter=0)
    rec = L.record(0).tobytes()
    h = synth.parse_header(rec)
    payload = rec[48:h["chan_corr_off"] + 2 * (64 + 64 + 64)]
    assert zlib.crc32(payload) & 0xFFFFFFFF == h["crc32"]


def test_zipf_routes():
    r = synth.zipf_routes(0, 512, 256, 8)
    assert r.shape == (512, 8)
    assert all(len(set(row)) == 8 for row in r)
    counts = np.bincount(r.ravel(), minlength=256)
    assert counts.max() > 10 * np.median(counts[counts > 0])


def test_bank_range_splits_agree():
    """A rank's records are the same bytes whatever the split, carry their
    global expert ids, and pass the engine's record check."""
    inter, lat, E = 64, 128, 6
    L = synth.moe_layer(3, hidden=lat, inter=inter, n_experts=E, top_k=2, shared_inter=0)
    cb = L.cb_base
    whole = synth.bank_range(5, L.layer, 0, E, cb, inter, lat)
    a = synth.bank_range(5, L.layer, 0, 2, cb, inter, lat)
    b = synth.bank_range(5, L.layer, 2, 4, cb, inter, lat)
    assert np.array_equal(np.concatenate([a, b]), whole)
    L.bank = whole.reshape(-1).copy()
    keep = []
    s = O._moe_struct(L, keep)
    for e in range(E):
        assert synth.parse_header(L.record(e))["expert_id"] == e
        assert O.lib().orc_record_check(O.C.byref(s), L.layer, e) == 0
    moved = whole.copy()
    synth.set_layer(moved, 9)
    assert all(synth.parse_header(r)["layer"] == 9 for r in moved)
    assert np.array_equal(moved[:, 48:], whole[:, 48:])
