"""Banks loaded straight from bank files (waste_cuda_vq_bank_load_file):
pread into pinned staging, uploads overlapping the reads, every header
checked — the device side of the engine's per-record reads
(src/model.c:1767-1795 bank_fetch, records at e * rec_bytes).

A layer loaded from its file computes exactly what the same records loaded
from memory compute; ranges of records load in separate calls; a file that
ends early and a record whose header does not match are refused."""
import os
import tempfile

import numpy as np
import pytest

from golden_cases import bits
from warp_b200 import synth

pytestmark = pytest.mark.gpu


def _route(L, rng):
    idx = rng.choice(L.n_experts, size=L.top_k, replace=False).astype(np.int32)
    w = rng.uniform(0.1, 0.5, size=L.top_k).astype(np.float32)
    return idx, w


def test_bank_from_file_matches_memory(cuda_lib):
    wb = cuda_lib
    A = synth.moe_layer(801, hidden=1024, inter=512, n_experts=48, top_k=6, shared_inter=0,
                        layer=70, cb_base=0)
    B = synth.derive_layer(A, 71, 802)              # the same records under layer 71
    wb.codebooks_load_f16(A.books_raw)
    wb.vq_bank_free(70)
    wb.vq_bank_free(71)
    wb.vq_bank_load(70, A.n_experts, A.rec_bytes, 0, A.n_experts, A.bank, A.inter, A.hidden)
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "experts-L71.bin")
        B.bank.tofile(path)
        half = B.n_experts // 2                      # two calls, two ranges
        wb.vq_bank_load_file(71, path, B.n_experts, B.rec_bytes, 0, half, B.inter, B.hidden)
        wb.vq_bank_load_file(71, path, B.n_experts, B.rec_bytes, half, B.n_experts - half,
                             B.inter, B.hidden)
    rng = np.random.default_rng(803)
    for t in range(3):
        idx, w = _route(A, rng)
        x = synth.activations(804 + t, A.hidden)[0]
        ya = wb.moe_experts(70, idx, w, x, A.hidden, A.inter)
        yb = wb.moe_experts(71, idx, w, x, A.hidden, A.inter)
        assert np.array_equal(bits(ya), bits(yb))
    wb.vq_bank_free(70)
    wb.vq_bank_free(71)


def test_bank_file_refusals(cuda_lib):
    wb = cuda_lib
    A = synth.moe_layer(811, hidden=256, inter=128, n_experts=8, top_k=2, shared_inter=0,
                        layer=72, cb_base=0)
    wb.codebooks_load_f16(A.books_raw)
    wb.vq_bank_free(72)
    with tempfile.TemporaryDirectory() as d:
        short = os.path.join(d, "short.bin")
        A.bank[: 5 * A.rec_bytes].tofile(short)        # 5 of 8 records
        with pytest.raises(wb.WasteCudaError) as e:
            wb.vq_bank_load_file(72, short, A.n_experts, A.rec_bytes, 0, 8, A.inter, A.hidden)
        assert e.value.rc == wb.E_ARG and "short read" in str(e.value)
        bad = os.path.join(d, "bad.bin")
        b = A.bank.copy()
        b[2 * A.rec_bytes + 4] ^= 0xFF                  # expert 2's layer field
        b.tofile(bad)
        wb.vq_bank_free(72)
        with pytest.raises(wb.WasteCudaError) as e:
            wb.vq_bank_load_file(72, bad, A.n_experts, A.rec_bytes, 0, 8, A.inter, A.hidden)
        assert e.value.rc == wb.E_RECORD
    wb.vq_bank_free(72)
