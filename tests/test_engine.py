"""The reference engine with this backend wired in (integration/), driven
through its public API (waste.h: waste_open, waste_eval) on the reference's
own test container (tests/golden/tiny_container: a Kimi-Linear at 1/18
scale, 3 MoE layers of 8 VQ3R experts, top-2).

integration/warp_cuda.patch adds the expert-path slots to the engine's
src/backend.c and, in src/model.c, the bank upload after load and the slot
calls before moe_layer's and moe_chunk's CPU expert loops
(src/model.c:2873, :3585). The same driver (integration/engine_run.c) runs
the unmodified reference engine (oracle/_ref) and the patched one, on a
prompt (one waste_eval of six tokens: a chunked prefill through moe_chunk)
and then greedy decode steps (moe_layer).

  * no device (this test): the patched engine's CUDA registration declines
    (the reference's contract, src/waste_backend.h:116-120), and its logits
    are the reference's bit for bit;
  * on a B200 (tests/test_engine_gpu.py): the backend registers, the
    experts run on the device, and the engine's outputs stay within
    tolerance of the reference.
"""
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ENGINE_RUN = os.path.join(ROOT, "integration", "_build", "engine_run")
CUDA_ENGINE = os.path.join(ROOT, "integration", "_build", "libwaste_engine_cuda.so")
REF_ENGINE = os.path.join(ROOT, "oracle", "_ref", "libwaste_ref.so")
CONTAINER = os.path.join(ROOT, "tests", "golden", "tiny_container")
PROMPT = [1, 5, 9, 77, 3, 12]
STEPS = 6

needs_engines = pytest.mark.skipif(
    not all(os.path.exists(p) for p in (ENGINE_RUN, CUDA_ENGINE, REF_ENGINE)),
    reason="integration/_build or oracle/_ref not built here")


def run_engine(lib, tmp_path, tag, env=None):
    """(build line, launches or None, tokens [evals], logits [evals][vocab])."""
    out = os.path.join(str(tmp_path), f"{tag}.bin")
    r = subprocess.run([ENGINE_RUN, lib, CONTAINER, out, str(STEPS)] + [str(t) for t in PROMPT],
                       capture_output=True, text=True, timeout=600,
                       env=dict(os.environ, **(env or {})))
    assert r.returncode == 0, r.stdout + r.stderr
    build = next(l for l in r.stdout.splitlines() if l.startswith("build:"))
    launches = None
    for l in r.stdout.splitlines():
        if l.startswith("cuda launches:"):
            launches = int(l.split(":")[1])
    raw = np.fromfile(out, dtype=np.int32)
    nev, vocab = int(raw[0]), int(raw[1])
    rows = raw[2:].reshape(nev, 1 + vocab)
    return build, launches, rows[:, 0].copy(), rows[:, 1:].copy().view(np.float32)


def _has_device():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@needs_engines
@pytest.mark.skipif(_has_device(), reason="declining is only observable without a device")
def test_patched_engine_declines_and_matches_bitwise(tmp_path):
    b_ref, _, tok_ref, lg_ref = run_engine(REF_ENGINE, tmp_path, "ref")
    b_cu, launches, tok_cu, lg_cu = run_engine(CUDA_ENGINE, tmp_path, "cuda")
    assert "CUDA" not in b_cu and b_cu == b_ref
    assert launches == 0
    assert np.array_equal(tok_ref, tok_cu)
    assert np.array_equal(lg_ref.view(np.uint32), lg_cu.view(np.uint32))


def test_patch_is_additions_only():
    """The patch adds lines and removes none, so the engine it applies to
    keeps every line of the reference's code path."""
    lines = open(os.path.join(ROOT, "integration", "warp_cuda.patch")).read().splitlines()
    removed = [l for l in lines if l.startswith("-") and not l.startswith("---")]
    assert not removed
    assert sum(l.startswith("+") and not l.startswith("+++") for l in lines) > 50
