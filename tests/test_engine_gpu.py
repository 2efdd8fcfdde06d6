"""The reference engine with the CUDA backend wired in (integration/), on a
B200, against the unmodified reference engine (oracle/_ref).

Two levels:
  * the public API (waste_open / waste_eval) on the reference's own test
    container: the patched engine registers the CUDA backend, its expert
    loops run on the device (the backend's launch count grows), and the
    greedy tokens match the reference's while the logits stay within 1e-4
    relative L2 (four decoder layers of fp32 arithmetic in between, so this
    is looser than the per-layer bound);
  * the same with every trunk matvec (the mvq_rows_f32 slot) on the device;
  * the engine's own moe_layer and moe_chunk at the Kimi-Linear-48B shape,
    reached through the oracle's harness compiled against the patched
    model.c: the route comes from the engine's CPU router in both engines
    (identical bits), and the layer outputs — routed experts through the
    moe_experts / moe_chunk_experts slots, the shared expert on the CPU —
    are within 2e-5 relative L2 of the reference's. 64-token chunks take
    the tensor-core path, 5-token chunks the lookup path; SiTU too.
"""
import numpy as np
import pytest

import oracle as O
from golden_cases import rel_l2
from test_engine import CUDA_ENGINE, REF_ENGINE, needs_engines, run_engine
from warp_b200 import synth

pytestmark = [pytest.mark.gpu, needs_engines]
TOL = 2e-5


def test_engine_public_api_on_device(tmp_path):
    b_ref, _, tok_ref, lg_ref = run_engine(REF_ENGINE, tmp_path, "ref")
    b_cu, launches, tok_cu, lg_cu = run_engine(CUDA_ENGINE, tmp_path, "cuda")
    assert "CUDA sm_100a" in b_cu, b_cu
    assert launches and launches > 0
    assert np.array_equal(tok_ref, tok_cu)
    worst = max(rel_l2(lg_cu[e], lg_ref[e]) for e in range(len(tok_ref)))
    assert worst < 1e-4, worst


def test_engine_trunk_on_device(tmp_path):
    """Every trunk matvec of the engine through the mvq_rows_f32 slot on the
    device (WASTE_CUDA_TRUNK_MIN=0 takes even the small ones): more of the
    backend's kernels run, and the tokens and logits still match."""
    _, _, tok_ref, lg_ref = run_engine(REF_ENGINE, tmp_path, "ref")
    _, l_exp, _, _ = run_engine(CUDA_ENGINE, tmp_path, "experts")
    b_cu, launches, tok_cu, lg_cu = run_engine(CUDA_ENGINE, tmp_path, "trunk",
                                               env={"WASTE_CUDA_TRUNK_MIN": "0"})
    assert "CUDA sm_100a" in b_cu
    assert launches > l_exp
    assert np.array_equal(tok_ref, tok_cu)
    worst = max(rel_l2(lg_cu[e], lg_ref[e]) for e in range(len(tok_ref)))
    assert worst < 1e-4, worst


def _pair(L, R):
    ref = O.RefMoe(L, max_tokens=64)
    cu = O.RefMoe(L, max_tokens=64, lib=R)
    assert R.refh_moe_upload(cu.h) == 1, "the backend declined the bank"
    return ref, cu


@pytest.mark.parametrize("act", [0, 1])
def test_engine_moe_layer_and_chunk_through_slots(cuda_lib, act):
    wb = cuda_lib
    R = O.engine_cuda()
    assert b"CUDA" in R.refh_backend_auto()
    L = synth.moe_layer(1234, layer=90, cb_base=0, act_situ=act)
    x = synth.activations(90 + act, L.hidden, T=64)
    ref, cu = _pair(L, R)
    try:
        n0 = wb.launch_count()
        for t in range(3):                       # decode: moe_layer
            o_r, i_r = ref.layer(x[t])
            o_c, i_c = cu.layer(x[t])
            assert np.array_equal(i_r, i_c)
            assert rel_l2(o_c, o_r) < TOL, t
        assert wb.launch_count() > n0
        for T in (64, 5):                        # prefill: moe_chunk
            c_r, r_r, w_r = ref.chunk(x[:T])
            c_c, r_c, w_c = cu.chunk(x[:T])
            assert np.array_equal(r_r, r_c)
            worst = max(rel_l2(c_c[t], c_r[t]) for t in range(T))
            assert worst < TOL, (T, worst)
        assert wb.device_errors() == 0
    finally:
        cu.close()
        ref.close()


def test_engine_kda_on_device(tmp_path):
    """The reference's test container has KDA layers (4 heads of 32): with
    the kda_step slot (on by default) and the conv and gated-norm slots
    switched on, the decoder's linear attention runs on the device — its
    recurrent state and conv rings held in HBM across tokens — and the
    tokens and logits still match the reference's."""
    _, _, tok_ref, lg_ref = run_engine(REF_ENGINE, tmp_path, "ref")
    _, l_off, tok_off, _ = run_engine(CUDA_ENGINE, tmp_path, "kda_off", env={"WASTE_CUDA_KDA": "0"})
    b_cu, launches, tok_cu, lg_cu = run_engine(
        CUDA_ENGINE, tmp_path, "kda_all",
        env={"WASTE_CUDA_KDA_CONV": "1", "WASTE_CUDA_KDA_NORM": "1"})
    assert "CUDA sm_100a" in b_cu
    # 3 KDA layers x (1 step + 3 convs + 1 norm) launches per decode step, at least
    assert launches >= l_off + 3 * 5 * (len(tok_ref) - 1)
    assert np.array_equal(tok_ref, tok_off)
    assert np.array_equal(tok_ref, tok_cu)
    worst = max(rel_l2(lg_cu[e], lg_ref[e]) for e in range(len(tok_ref)))
    assert worst < 1e-4, worst


def test_engine_snapshot_with_state_on_device(tmp_path):
    """waste_state_save / waste_state_reset / waste_state_load with the KDA
    state and conv rings in HBM: the patched engine pulls them before the
    save and pushes them after the reset and the load, so the prompt after
    the reset repeats eval 0 bit for bit, and the decode after the load
    repeats the uninterrupted run's, in both engines."""
    env = {"WASTE_CUDA_KDA_CONV": "1", "WASTE_CUDA_KDA_NORM": "1"}
    from test_engine import STEPS
    half = STEPS // 2
    for lib, tag in ((REF_ENGINE, "ref"), (CUDA_ENGINE, "cuda")):
        _, _, tok_u, lg_u = run_engine(lib, tmp_path, tag + "_u", env=env)
        _, _, tok_s, lg_s = run_engine(
            lib, tmp_path, tag + "_s",
            env=dict(env, ENGINE_RUN_STATE=str(tmp_path / f"{tag}.state")))
        assert len(tok_s) == len(tok_u) + 1
        assert np.array_equal(lg_s[1 + half].view(np.uint32), lg_u[0].view(np.uint32))
        assert np.array_equal(lg_s[2 + half:].view(np.uint32), lg_u[1 + half:].view(np.uint32))
        assert np.array_equal(lg_s[:1 + half].view(np.uint32), lg_u[:1 + half].view(np.uint32))


def test_engine_whole_layers_on_device(tmp_path):
    """A container from warp_b200.synth.write_container (F32 router, Q8G
    shared expert, KDA and MLA layers) at a small width: the patched engine
    runs each MoE layer whole in one call (router, experts, shared expert:
    the moe_layer slot) and each KDA attention layer whole in one call (the
    kda_layer slot); tokens match the unmodified engine's and logits stay
    within 1e-4, as they do with either slot switched off."""
    import os
    import subprocess
    from test_engine import ENGINE_RUN
    cdir = str(tmp_path / "c")
    synth.write_container(cdir, seed=3, hidden=256, layers=5, dense_inter=512, moe_inter=128,
                          experts=16, top_k=4, kda_heads=4, kda_dim=64, mla_heads=4, qk_nope=32,
                          qk_rope=16, v_head=32, kv_lora=64, vocab=1024, full_attn=(3,))

    def run(lib, tag, env=None):
        out = str(tmp_path / f"{tag}.bin")
        r = subprocess.run([ENGINE_RUN, lib, cdir, out, "6", "1", "17", "42", "99"],
                           capture_output=True, text=True, timeout=600,
                           env=dict(os.environ, **(env or {})))
        assert r.returncode == 0, r.stdout + r.stderr
        n = [int(l.split(":")[1]) for l in r.stdout.splitlines() if l.startswith("cuda launches")]
        raw = np.fromfile(out, dtype=np.int32)
        rows = raw[2:].reshape(int(raw[0]), 1 + int(raw[1]))
        return (n[0] if n else None), rows[:, 0].copy(), rows[:, 1:].copy().view(np.float32)

    _, tok_ref, lg_ref = run(REF_ENGINE, "ref")
    l_whole, tok_w, lg_w = run(CUDA_ENGINE, "whole")
    l_split, tok_s, lg_s = run(CUDA_ENGINE, "split", {"WASTE_CUDA_MOE_LAYER": "0",
                                                      "WASTE_CUDA_KDA_LAYER": "0"})
    _, tok_k, lg_k = run(CUDA_ENGINE, "kda_only", {"WASTE_CUDA_MOE_LAYER": "0"})
    for tok, lg in ((tok_w, lg_w), (tok_s, lg_s), (tok_k, lg_k)):
        assert np.array_equal(tok_ref, tok)
        assert max(rel_l2(lg[e], lg_ref[e]) for e in range(len(tok_ref))) < 1e-4
    assert l_whole != l_split                      # the paths launch different kernels
