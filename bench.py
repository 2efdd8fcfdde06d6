#!/usr/bin/env python
"""bench.py — MoE decode throughput at the Kimi-Linear-48B shape on B200.

Workload (extended to a whole decode step's MoE work):
one step is ONE token through the 26 MoE layers of a Kimi-Linear-48B-shaped
model (27 layers, layer 0 dense), chained the way the decode step chains
them (src/model.c:3927-3945): each layer's MoE block takes the residual
stream h the previous layer left, normalises it (rmsnorm with the layer's
post-attention weight), runs the layer = router (256 experts, F32) ->
sigmoid top-8 with renorm and routed scale 2.446 -> 8 routed experts whose
gate/up/down weights are 3-bit residual VQ (3 x 256-entry codebooks over
8-dim vectors) -> router-order reduce -> + one Q8G shared expert, and adds
the result to h, which is the next layer's input. hidden 2304, expert
intermediate 1024. All 26 layers' 256 experts are resident in HBM (26 x 683
MB); the step's first h is seeded synthetic (bf16-valued N(0,1)). A step
touches ~803 MB, far more than the 126 MB L2, so no L2 flush is needed
between steps.

Also measured: the config-1 VQ3R matvec (4096 x 4096) as a batched launch
over 32 distinct matrices (203 MB of indices), in HBM GB/s; and, at one GPU,
config 5 (`engine_step`, see `--workload engine` below) — the whole decode
step through the reference engine's waste.h with this backend wired in.

`--impl reference` times the reference engine's own moe_layer (compiled
from the reference sources into oracle/_ref) on this host's cores, same
metric and config.

Multi-GPU (torchrun, --gpus N > 1): expert parallel — each rank holds a
contiguous 1/N of every layer's experts (the router and shared expert are
replicated) and contributes one token per step, so a step decodes N tokens;
the routed tokens and partial sums cross NVLink inside the library's own
kernels (peer-memory mailboxes; NCCL as the fallback). Per-GPU work stays
~K expert-token pairs per layer (weak scaling). `--parallel replicas`
instead runs N independent copies of the single-GPU decode.

`--workload k3` measures config 4 instead: one K3-class MoE layer (hidden
7168, 512 experts, top-16) at global batches 1/16/64, expert parallel over
the N GPUs.

`--workload engine` measures config 5: the whole decode step through the
reference engine's public API (waste_open / waste_eval), built with this
backend wired in (integration/), on a synthetic Kimi-Linear-48B-shaped
container (27 layers: a dense layer, 21 KDA and 6 MLA layers, 26 MoE
layers of 256 experts; ~19 GB, written once by warp_b200.synth into
--container, default /dev/shm/warp_c5). Every slot is live: the trunk
matvecs, the KDA steps and the expert loops run on the device, MLA and
the router on the host. Tokens/s is the wall clock of waste_eval per
decode step (host API, copies included, so value and e2e coincide); the
unmodified reference engine on the same container is the CPU baseline.
Single GPU (the engine is one process).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = ("MoE decode tok/s (26 chained VQ3R MoE blocks: rmsnorm, MoE layer, residual; "
          "Kimi-Linear-48B shape, batch 1)")
UNIT = "tok/s"
HIDDEN, INTER, EXPERTS, TOPK, SHARED = 2304, 1024, 256, 8, 1024
MOE_LAYERS = 26
SEED = 1234


def layer_bytes():
    """Algorithmic bytes one token reads in one layer: the 8 routed experts'
    index streams and row scales, the Q8G shared expert, the F32 router,
    the layer's codebooks and x in / y out."""
    from warp_b200 import synth
    idx = 2 * synth.index_bytes(INTER, HIDDEN, 3) + synth.index_bytes(HIDDEN, INTER, 3)
    scales = 2 * (2 * INTER + HIDDEN)
    routed = TOPK * (idx + scales)
    ng_h, ng_s = (HIDDEN + 127) // 128, (SHARED + 127) // 128
    shared = 2 * SHARED * ng_h * 128 + HIDDEN * ng_s * 128 + 2 * (2 * SHARED * ng_h + HIDDEN * ng_s)
    router = EXPERTS * HIDDEN * 4
    books = 9 * 256 * 8 * 4
    return routed + shared + router + books + 2 * HIDDEN * 4


# DRAM traffic of one gateup_kernel launch (dram__bytes_read.sum +
# dram__bytes_write.sum), from one ncu capture of this bench's workload
# (profiles/gateup_kernel_kimi_linear_decode.txt): the algorithmic bytes plus
# the deliberate L2 prefetch of the chosen experts' down streams.
GATEUP_TRAFFIC_BYTES = 21_357_184     # mean of the two captured launches


def gateup_bytes():
    """Algorithmic bytes of one gate/up launch (K experts, one token)."""
    from warp_b200 import synth
    return 2 * TOPK * synth.index_bytes(INTER, HIDDEN, 3) + HIDDEN * 4 + 2 * 3 * 256 * 8 * 4


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class Clocks:
    """nvidia-smi sampling during the timed region (200 ms period)."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.path = tempfile.mktemp(prefix="clocks_", suffix=".csv")
        self.device = device
        self.proc = None

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f,
                stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup(n_gpus):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}")
    return rank, world, local


# ---------------------------------------------------------------- reference

def run_reference(args):
    import oracle as O
    from warp_b200 import synth
    rank, world, _ = dist_setup(args.gpus)
    if rank != 0:
        return 0
    ncores = os.cpu_count() or 1
    base = synth.moe_layer(SEED)
    xs = synth.activations(SEED + 1, HIDDEN, T=64)
    norms = [synth.norm_weight(SEED + 200 + L, HIDDEN) for L in range(1, MOE_LAYERS + 1)]
    if O.ref_available():
        layers = [O.RefMoe(base, max_tokens=1, threads=0),
                  O.RefMoe(synth.derive_layer(base, 2, SEED + 2), max_tokens=1, threads=0)]
        kind, cores = "reference", O.ref().refh_pool_threads()
        backend = layers[0].backend.decode()
        rmsnorm = O.ref_rmsnorm
        step_layer = lambda L, x: layers[L % 2].layer(x)[0]
    else:
        ders = [base, synth.derive_layer(base, 2, SEED + 2)]
        kind, cores, backend = "port", 1, "restatement"
        rmsnorm = O.rmsnorm
        step_layer = lambda L, x: O.moe_layer(ders[L % 2], x)[0]

    def step(k):
        # the decode step's chain (src/model.c:3927-3945): h += moe(rmsnorm(h))
        h = xs[k % 64]
        for L in range(MOE_LAYERS):
            h = h + step_layer(L, rmsnorm(h, norms[L], synth.NORM_EPS))

    for k in range(args.warmup):
        step(k)
    t0 = time.perf_counter()
    for k in range(args.steps):
        step(args.warmup + k)
    dt = time.perf_counter() - t0
    v = args.steps / dt
    sample = (f"{args.steps} tokens x {MOE_LAYERS} chained MoE blocks through the reference's "
              f"waste_rmsnorm and moe_layer ({backend}, {cores} threads), h += output; banks "
              f"alternate between 2 resident layers (683 MB each, larger than the host caches)")
    line = {"metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3 / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "impl": "reference",
            "config": {"workload": "kimi_linear_48b_moe_decode", "hidden": HIDDEN,
                       "moe_inter": INTER, "experts": EXPERTS, "top_k": TOPK,
                       "moe_layers": MOE_LAYERS, "global_batch": 1, "parallelism": "cpu"},
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": cores, "kind": kind,
                             "sample": sample},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    for L in (layers if kind == "reference" else []):
        L.close()
    return 0


def cpu_baseline(budget_s=10.0):
    """The reference CPU path on this host, bounded sample (rank 0, N=1)."""
    import oracle as O
    from warp_b200 import synth
    base = synth.moe_layer(SEED)
    xs = synth.activations(SEED + 1, HIDDEN, T=16)
    if O.ref_available():
        rm = O.RefMoe(base, max_tokens=1, threads=0)
        run, kind, cores = rm.layer, "reference", O.ref().refh_pool_threads()
    else:
        rm, kind, cores = None, "port", 1
        run = lambda x: O.moe_layer(base, x)
    run(xs[0])
    t0 = time.perf_counter()
    run(xs[1])
    per = max(time.perf_counter() - t0, 1e-4)
    n = max(2, min(400, int(budget_s / per)))
    t0 = time.perf_counter()
    for i in range(n):
        run(xs[i % 16])
    dt = (time.perf_counter() - t0) / n
    if rm is not None:
        rm.close()
    return {"value": 1.0 / (dt * MOE_LAYERS), "unit": UNIT, "cores": cores, "kind": kind,
            "sample": f"{n} single-token MoE layer calls ({dt * 1e3:.2f} ms each) at the "
                      f"Kimi-Linear shape, scaled to {MOE_LAYERS} layers per token"}


def engine_slot_path(base, budget_s=3.0):
    """The drop-in as an engine binds it: the reference engine patched with
    this backend (integration/), its own moe_layer at the Kimi-Linear shape
    through the oracle's harness. Per layer: the engine's CPU router, the
    routed experts through the moe_experts slot (host buffers: x, route and
    weights in, ysum out, one synchronisation), the shared expert on the
    CPU. Returns tok/s for 26 such layers, the per-layer time, and the time
    of the slot call alone (waste_cuda_moe_experts) on the same layer."""
    import oracle as O
    import warp_b200 as wb
    from warp_b200 import synth
    R = O.engine_cuda()
    if R is None:
        return {"unavailable": "integration/_build/libwaste_engine_cuda.so is not built"}
    backend = R.refh_backend_auto().decode()
    L = synth.derive_layer(base, 100, SEED + 300)
    rm = O.RefMoe(L, max_tokens=1, lib=R)
    try:
        if not R.refh_moe_upload(rm.h):
            return {"unavailable": "the CUDA backend declined the bank"}
        xs = synth.activations(SEED + 301, HIDDEN, T=16)
        for i in range(3):
            rm.layer(xs[i])
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < budget_s:
            rm.layer(xs[n % 16])
            n += 1
        per = (time.perf_counter() - t0) / n
        routes = [O.moe_layer(L, xs[i])[1:] for i in range(4)]
        for i in range(4):
            wb.moe_experts(100, routes[i][0], routes[i][1], xs[i], HIDDEN, INTER)
        m, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < budget_s / 2:
            i = m % 4
            wb.moe_experts(100, routes[i][0], routes[i][1], xs[i], HIDDEN, INTER)
            m += 1
        slot = (time.perf_counter() - t0) / m
    finally:
        rm.close()
    return {"value": 1.0 / (per * MOE_LAYERS), "unit": UNIT, "ms_per_layer": per * 1e3,
            "slot_ms_per_layer": slot * 1e3, "layer_calls": n, "engine_backend": backend,
            "cpu_threads": int(R.refh_pool_threads()),
            "h2d_bytes_per_step": MOE_LAYERS * (HIDDEN + 2 * TOPK) * 4,
            "d2h_bytes_per_step": MOE_LAYERS * (HIDDEN + 1) * 4,
            "path": "the reference engine's moe_layer with integration/warp_cuda.patch: CPU "
                    "router and shared expert, routed experts through the moe_experts slot"}


# ---------------------------------------------------------------- this repo

def run_warp(args):
    import torch
    import warp_b200 as wb
    from warp_b200 import synth

    rank, world, local = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    wb.init(local)
    dev = torch.device("cuda", local)
    ep_mode = world > 1 and args.parallel == "ep"
    first, count = 0, EXPERTS
    if ep_mode:
        from warp_b200 import ep
        ep.setup(rank, world)
        first, count = ep.ep_range(EXPERTS, rank, world)

    # ---- resident layers (this rank's experts)
    base = synth.moe_layer(SEED)
    nL = args.layers
    for L in range(1, nL + 1):
        lay = base if L == 1 else synth.derive_layer(base, L, SEED + L)
        wb.vq_bank_free(L)
        if L == 1:
            wb.codebooks_load_f16(base.books_raw)
        wb.vq_bank_load(L, lay.n_experts, lay.rec_bytes, first, count,
                        lay.bank[first * lay.rec_bytes:], lay.inter, lay.hidden, lay.stages)
        wb.moe_trunk_load(L, lay.n_experts, lay.hidden, lay.top_k, lay.renorm,
                          lay.routed_scale, lay.router, lay.bias, lay.shared_inter, lay.sh)
        wb.moe_norm_load(L, synth.norm_weight(SEED + 200 + L, HIDDEN), synth.NORM_EPS)
        del lay
    ntok = 4
    # the step's first h per token slot; the layers' outputs alternate
    # between two buffers, each layer reading the one the last layer wrote
    xs_h = synth.activations(SEED + 100 + rank, HIDDEN, T=ntok)
    xs = torch.from_numpy(xs_h).to(dev)
    hbuf = torch.empty((2, HIDDEN), dtype=torch.float32, device=dev)
    idx = torch.empty((nL, TOPK), dtype=torch.int32, device=dev)
    w = torch.empty((nL, TOPK), dtype=torch.float32, device=dev)
    s = torch.cuda.Stream(device=dev)

    def h_in(t, L):
        return xs[t].data_ptr() if L == 0 else hbuf[(L - 1) % 2].data_ptr()

    def step_direct(t):
        for L in range(nL):
            if ep_mode:
                ep.moe_block_dev(L + 1, 1, h_in(t, L), hbuf[L % 2].data_ptr(),
                                 idx[L].data_ptr(), w[L].data_ptr(), s.cuda_stream)
            else:
                wb.moe_block_dev(L + 1, 1, h_in(t, L), hbuf[L % 2].data_ptr(),
                                 idx[L].data_ptr(), w[L].data_ptr(), s.cuda_stream)

    with torch.cuda.stream(s):
        for k in range(max(args.warmup, 1)):
            step_direct(k % ntok)
    torch.cuda.synchronize()

    # ---- one CUDA graph per token slot
    def capture(t):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s, capture_error_mode="thread_local"):
            step_direct(t)
        return g

    graphs = []           # the only references: released before the communicators go
    launches_per_step = None
    try:
        for t in range(ntok):
            c0 = wb.launch_count()
            graphs.append(capture(t))
            launches_per_step = wb.launch_count() - c0
        use_graphs = True
    except Exception as e:  # direct launches still measure the same kernels
        print(f"graph capture unavailable: {e}", file=sys.stderr)
        graphs, use_graphs = [], False
        launches_per_step = 4 * nL

    def step(k):
        if use_graphs:
            graphs[k % ntok].replay()
        else:
            step_direct(k % ntok)

    clocks = Clocks(local)
    clocks.start()
    with torch.cuda.stream(s):
        for k in range(args.warmup):
            step(k)
    torch.cuda.synchronize()
    # Let clocks settle for ~0.5 s. Every rank runs the SAME number of steps
    # (an expert-parallel step holds collectives): one step is timed, the
    # slowest rank's time sets the count.
    t1 = time.perf_counter()
    with torch.cuda.stream(s):
        step(0)
    s.synchronize()
    t_step = torch.tensor([time.perf_counter() - t1], dtype=torch.float64, device=dev)
    if dist:
        dist.all_reduce(t_step, op=dist.ReduceOp.MAX)
    n_settle = max(1, min(2000, int(0.5 / max(float(t_step.item()), 1e-5))))
    with torch.cuda.stream(s):
        for k in range(n_settle):
            step(k)
            if k % 64 == 63:
                s.synchronize()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    with torch.cuda.stream(s):
        for k in range(args.steps):
            step(k)
    e1.record(s)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ck = clocks.stop()
    ms = e0.elapsed_time(e1)
    if dist:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / args.steps
    value = world * args.steps / (ms / 1e3)

    # ---- end to end through the public entry points, host buffers: each
    # layer's h copied in from host memory and its h_out copied back, the
    # next layer reading what the last one returned (an engine that runs
    # attention on the host between the MoE blocks)
    h_host = [np.ascontiguousarray(xs_h[t]) for t in range(ntok)]
    hb_host = [np.empty(HIDDEN, np.float32), np.empty(HIDDEN, np.float32)]
    if ep_mode:
        h_pin = torch.empty((2, HIDDEN), dtype=torch.float32).pin_memory()
        hd = torch.empty((2, HIDDEN), dtype=torch.float32, device=dev)

        def e2e_layer(t, L):
            src = h_host[t] if L == 0 else hb_host[(L - 1) % 2]
            with torch.cuda.stream(s):
                h_pin[0].copy_(torch.from_numpy(src))
                hd[0].copy_(h_pin[0], non_blocking=True)
                ep.moe_block_dev(L + 1, 1, hd[0].data_ptr(), hd[1].data_ptr(), idx[L].data_ptr(),
                                 w[L].data_ptr(), s.cuda_stream)
                h_pin[1].copy_(hd[1], non_blocking=True)
            s.synchronize()
            hb_host[L % 2][:] = h_pin[1].numpy()
    else:
        # the C entry point with caller-owned host buffers (what an engine
        # in C passes): the library copies h to the device and h_out, the
        # route and the weights back on every call; addresses taken once
        h_addr = [a.ctypes.data for a in h_host]
        hb_addr = [a.ctypes.data for a in hb_host]
        i_host = np.empty(TOPK, np.int32)
        w_host = np.empty(TOPK, np.float32)
        i_a, w_a = i_host.ctypes.data, w_host.ctypes.data
        block_call = wb.load_library().waste_cuda_moe_block

        def e2e_layer(t, L):
            rc = block_call(L + 1, h_addr[t] if L == 0 else hb_addr[(L - 1) % 2],
                            hb_addr[L % 2], i_a, w_a)
            if rc:
                wb._check(rc)
    for L in range(nL):
        e2e_layer(0, L)
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for k in range(args.steps):
        for L in range(nL):
            e2e_layer(k % ntok, L)
    e2e_s = time.perf_counter() - t0
    if dist:
        t = torch.tensor([e2e_s], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    # per layer: h in; h_out, the route, the weights and the error word back
    # (the library's result block: hidden + 2 x 64 + 4 words)
    e2e = {"value": world * args.steps / e2e_s, "unit": UNIT,
           "h2d_bytes_per_step": nL * HIDDEN * 4,
           "d2h_bytes_per_step": nL * ((HIDDEN + 2 * 64 + 4) * 4 if not ep_mode
                                       else HIDDEN * 4)}

    # ---- parity, outside the timed region: this rank's own token through
    # layer 1's MoE block against the oracle (routes bit-exact, the MoE part
    # within 2e-5 relative L2), so a multi-GPU run carries its own evidence
    parity = None
    if not args.no_parity:
        import oracle as O
        nw1 = synth.norm_weight(SEED + 201, HIDDEN)
        hout = torch.empty((1, HIDDEN), dtype=torch.float32, device=dev)
        pi = torch.empty((1, TOPK), dtype=torch.int32, device=dev)
        pw = torch.empty((1, TOPK), dtype=torch.float32, device=dev)
        torch.cuda.synchronize()
        if ep_mode:
            ep.moe_block_dev(1, 1, xs[0].data_ptr(), hout.data_ptr(), pi.data_ptr(),
                             pw.data_ptr(), s.cuda_stream)
        else:
            wb.moe_block_dev(1, 1, xs[0].data_ptr(), hout.data_ptr(), pi.data_ptr(),
                             pw.data_ptr(), s.cuda_stream)
        torch.cuda.synchronize()
        derr = wb.device_errors()
        h0 = xs_h[0]
        ro, ri, _ = O.moe_block(base, h0, nw1, synth.NORM_EPS)
        got = hout.cpu().numpy()[0]
        d, r = (got - h0).astype(np.float64), (ro - h0).astype(np.float64)
        rel = float(np.linalg.norm(d - r) / max(np.linalg.norm(r), 1e-30))
        same = bool(np.array_equal(pi.cpu().numpy()[0], ri)) and derr == 0
        if dist:
            t = torch.tensor([rel, 0.0 if same else 1.0], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            rel, same = float(t[0].item()), t[1].item() == 0.0
        parity = {"ok": bool(same and rel < 2e-5), "worst_rel_l2": rel, "tolerance": 2e-5,
                  "routes_bit_exact": same,
                  "checked": f"layer 1 MoE block (rmsnorm, layer, residual) of one token per "
                             f"rank on {world} rank(s), against the oracle (max over ranks)"}

    # ---- per-kernel times (phase timers): a GPU-side sleep holds the stream
    # while the host queues the launches, so each event pair brackets kernel
    # time rather than host launch gaps. Kept under the launch-queue depth.
    prof_steps = max(1, min(args.steps, 700 // (12 * nL) or 1))
    wb.profile(True)
    with torch.cuda.stream(s):
        torch.cuda._sleep(int(2e6 * nL * prof_steps))      # ~1 ms per layer-call at 2 GHz
        for k in range(prof_steps):
            step_direct(k % ntok)
    torch.cuda.synchronize()
    ph = wb.profile_read()
    wb.profile(False)
    gu_ms, gu_n = ph["gateup"]
    gu_avg = gu_ms / max(gu_n, 1)
    peak, peak_src = peaks()
    achieved = gateup_bytes() / (gu_avg / 1e3) / 1e9
    tot = sum(v[0] for v in ph.values())
    kernels = {k: {"avg_us": (v[0] / max(v[1], 1)) * 1e3, "launches": v[1],
                   "share": v[0] / tot if tot else None} for k, v in ph.items() if v[1]}

    # ---- config 1: VQ3R matvec 4096 x 4096, 32 distinct matrices per launch
    matvec = None
    if not args.decode_only:
        G, M, N = 32, 4096, 4096
        rng = np.random.default_rng(SEED + 7)
        raw = synth.codebooks(rng, 3)
        wb.codebooks_load_f16(raw)
        mats = [synth.random_matrix(rng, M, N) for _ in range(G)]
        d_idx = torch.from_numpy(np.stack([m[0] for m in mats])).to(dev)
        d_sc = torch.from_numpy(np.stack([m[1].view(np.int16) for m in mats])).to(dev)
        d_x = torch.from_numpy(synth.activations(SEED + 8, N, T=G)).to(dev)
        d_y = torch.empty((G, M), dtype=torch.float32, device=dev)
        ptrs = ([d_idx[g].data_ptr() for g in range(G)], [d_sc[g].data_ptr() for g in range(G)],
                [d_x[g].data_ptr() for g in range(G)], [d_y[g].data_ptr() for g in range(G)])
        mv_iters = max(args.steps, 10)
        for _ in range(3):
            wb.vq_matvec_dev(*ptrs, M, N, 0, 3, s.cuda_stream)
        torch.cuda.synchronize()
        # The launches are queued behind a GPU-side sleep that outlasts the host's
        # enqueue time (the Python wrapper builds its pointer tables per call), so
        # the events bracket back-to-back device work only.
        m0, m1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(s):
            torch.cuda._sleep(int(2e8))                  # ~0.1 s at 2 GHz
            m0.record(s)
            for _ in range(mv_iters):
                wb.vq_matvec_dev(*ptrs, M, N, 0, 3, s.cuda_stream)
            m1.record(s)
        torch.cuda.synchronize()
        wb.profile(True)
        with torch.cuda.stream(s):
            torch.cuda._sleep(int(1e8))
            for _ in range(10):
                wb.vq_matvec_dev(*ptrs, M, N, 0, 3, s.cuda_stream)
        torch.cuda.synchronize()
        mph = wb.profile_read()
        wb.profile(False)
        mv_ms = m0.elapsed_time(m1) / mv_iters
        mv_bytes = G * (synth.index_bytes(M, N, 3) + 2 * M + 4 * N + 4 * M) + 3 * 256 * 8 * 4
        mv_tiles_avg = mph["matvec"][0] / max(mph["matvec"][1], 1)
        matvec = {"workload": "vq3r_matvec_4096x4096_x32", "GBps": mv_bytes / (mv_ms / 1e3) / 1e9,
                  "frac": mv_bytes / (mv_ms / 1e3) / 1e9 / peak, "ms_per_launch": mv_ms,
                  "gather_kernel_GBps": G * synth.index_bytes(M, N, 3) / (mv_tiles_avg / 1e3) / 1e9,
                  "bytes_per_launch": mv_bytes, "kernel": "plain tables"}
        # the same 32 matrices with interleaved table copies: each matrix's
        # copy-select stream is written once (untimed, as at load); the
        # stream's bytes are read on top of the algorithmic ones
        sel_res = {}
        for copies in (2, 4):
            nb = wb.vq_sel_bytes(M, N, 3, copies)
            d_sel = torch.empty((G, nb), dtype=torch.uint8, device=dev)
            for g in range(G):
                wb.vq_sel_build_dev(d_idx[g].data_ptr(), d_sel[g].data_ptr(), M, N, 3, copies,
                                    s.cuda_stream)
            sptr = [d_sel[g].data_ptr() for g in range(G)]
            scall = lambda: wb.vq_matvec_sel_dev(ptrs[0], sptr, ptrs[1], ptrs[2], ptrs[3], M, N, 0,
                                                 3, copies, s.cuda_stream)
            for _ in range(3):
                scall()
            torch.cuda.synchronize()
            with torch.cuda.stream(s):
                torch.cuda._sleep(int(2e8))
                m0.record(s)
                for _ in range(mv_iters):
                    scall()
                m1.record(s)
            torch.cuda.synchronize()
            sms = m0.elapsed_time(m1) / mv_iters
            sel_res[copies] = {"GBps": mv_bytes / (sms / 1e3) / 1e9,
                               "frac": mv_bytes / (sms / 1e3) / 1e9 / peak, "ms_per_launch": sms,
                               "select_bytes_per_launch": G * nb}
            del d_sel
        matvec["table_copies"] = sel_res
        best = max(sel_res, key=lambda c: sel_res[c]["GBps"])
        if sel_res[best]["GBps"] > matvec["GBps"]:
            matvec.update(GBps=sel_res[best]["GBps"], frac=sel_res[best]["frac"],
                          ms_per_launch=sel_res[best]["ms_per_launch"],
                          kernel=f"{best} interleaved table copies (copy-select stream)")
        # the same shape in the VQ4P format (four 64-entry stages, 6-bit indices
        # packed four to three bytes: the same index bytes), bit-exact to the
        # reference; a separate line, since it is another container format
        del d_idx
        raw4 = synth.codebooks(rng, 4, entries=synth.ENTRIES_VQ4P)
        wb.codebooks_load_f16(raw4)
        mats4 = [synth.random_matrix(rng, M, N, stages=4) for _ in range(G)]
        d_idx4 = torch.from_numpy(np.stack([m[0] for m in mats4])).to(dev)
        d_sc4 = torch.from_numpy(np.stack([m[1].view(np.int16) for m in mats4])).to(dev)
        p4 = ([d_idx4[g].data_ptr() for g in range(G)], [d_sc4[g].data_ptr() for g in range(G)],
              ptrs[2], ptrs[3])
        pcall = lambda: wb.vq4p_matvec_dev(*p4, M, N, 0, s.cuda_stream)
        for _ in range(3):
            pcall()
        torch.cuda.synchronize()
        with torch.cuda.stream(s):
            torch.cuda._sleep(int(2e8))
            m0.record(s)
            for _ in range(mv_iters):
                pcall()
            m1.record(s)
        torch.cuda.synchronize()
        p_ms = m0.elapsed_time(m1) / mv_iters
        p_bytes = G * (synth.index_bytes(M, N, 4) + 2 * M + 4 * N + 4 * M) + 4 * 64 * 8 * 4
        exact = None
        if not args.no_parity:       # matrix 0 against the oracle, outside the timing
            import oracle as O
            y4 = d_y[0].cpu().numpy()
            y4o = O.vq4p_matvec(mats4[0][0], mats4[0][1],
                                synth.activations(SEED + 8, N, T=G)[0], M, N,
                                synth.flush_f16(raw4), 0, fma=1)
            exact = bool(np.array_equal(y4.view(np.uint32), y4o.view(np.uint32)))
        matvec["vq4p"] = {"workload": "vq4p_matvec_4096x4096_x32", "ms_per_launch": p_ms,
                          "GBps": p_bytes / (p_ms / 1e3) / 1e9,
                          "frac": p_bytes / (p_ms / 1e3) / 1e9 / peak,
                          "bytes_per_launch": p_bytes, "launches_per_call": 2,
                          "bit_exact_vs_oracle": exact}
        del d_idx4, d_sc4

    # ---- config 3: prefill, 512 tokens with Zipf(1.1) routes, one layer (layer
    # 1's bank), on the tensor cores; the lookup path (8 host-slot chunks of 64
    # tokens, copies included) timed beside it
    prefill = None
    if not ep_mode and not args.decode_only:
        PT = 512
        route = synth.zipf_routes(SEED + 9, PT, EXPERTS, TOPK).astype(np.int32)
        rw = np.random.default_rng(SEED + 10).uniform(0.05, 0.6, size=route.shape).astype(np.float32)
        px = synth.activations(SEED + 11, HIDDEN, T=PT)
        d_r, d_rw = torch.from_numpy(route).to(dev), torch.from_numpy(rw).to(dev)
        d_px = torch.from_numpy(px).to(dev)
        d_po = torch.empty((PT, HIDDEN), dtype=torch.float32, device=dev)
        wb.codebooks_load_f16(base.books_raw)
        call = lambda: wb.moe_prefill_dev(1, PT, TOPK, d_r.data_ptr(), d_rw.data_ptr(),
                                          d_px.data_ptr(), d_po.data_ptr(), s.cuda_stream)
        for _ in range(3):
            call()
        torch.cuda.synchronize()
        p_iters = 10
        p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(s):
            torch.cuda._sleep(int(2e7))
            p0.record(s)
            for _ in range(p_iters):
                call()
            p1.record(s)
        torch.cuda.synchronize()
        p_ms = p0.elapsed_time(p1) / p_iters
        flops = 2.0 * PT * TOPK * 3 * INTER * HIDDEN
        touched = int(np.unique(route).size)
        os.environ["WASTE_CUDA_PREFILL_TC"] = "0"
        wb.moe_chunk_experts(1, route[:64], rw[:64], px[:64], HIDDEN, INTER)
        t0 = time.perf_counter()
        for c in range(PT // 64):
            wb.moe_chunk_experts(1, route[64 * c:64 * c + 64], rw[64 * c:64 * c + 64],
                                 px[64 * c:64 * c + 64], HIDDEN, INTER)
        lookup_ms = (time.perf_counter() - t0) * 1e3
        del os.environ["WASTE_CUDA_PREFILL_TC"]
        pk = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))) if os.path.exists(
            os.path.join(ROOT, "MEASURED_PEAKS.json")) else {}
        tpeak = float(pk.get("bf16_tflops", 1590.0))
        prefill = {"workload": "kimi_linear_moe_prefill_512tok_zipf1.1", "tokens": PT,
                   "experts_touched": touched, "ms_per_layer": p_ms,
                   "tok_per_s": PT / (p_ms / 1e3),
                   "algorithmic_tflops": flops / (p_ms / 1e3) / 1e12,
                   "tensor_peak_tflops": tpeak,
                   "frac_of_tensor_peak": flops / (p_ms / 1e3) / 1e12 / tpeak,
                   "mma_tflops_issued": 3 * flops / (p_ms / 1e3) / 1e12,
                   "weight_bytes": touched * synth.record_bytes(INTER, HIDDEN, 3),
                   "weight_GBps": touched * synth.record_bytes(INTER, HIDDEN, 3) / (p_ms / 1e3) / 1e9,
                   "lookup_path_ms_per_layer": lookup_ms,
                   "speedup_vs_lookup": lookup_ms / p_ms}

    # ---- the trunk matvec (the mvq_rows_f32 slot) at the Kimi-Linear
    # lm_head shape: 163840 x 2304 Q8G, 383 MB read once per token
    trunk = None
    if not args.decode_only:
        VOCAB = 163840
        rng = np.random.default_rng(SEED + 12)
        raw, sc, rb = synth.trunk_tensor(rng, VOCAB, HIDDEN, 8)
        dW = torch.from_numpy(raw).to(dev)
        ds = torch.from_numpy(sc.view(np.int16)).to(dev)
        del raw, sc
        dx = torch.from_numpy(synth.activations(SEED + 13, HIDDEN)[0]).to(dev)
        dy = torch.empty((VOCAB,), dtype=torch.float32, device=dev)
        call = lambda: wb.mvq_rows_dev(dy.data_ptr(), dW.data_ptr(), ds.data_ptr(), dx.data_ptr(),
                                       0, VOCAB, HIDDEN, 128, 8, rb, s.cuda_stream)
        for _ in range(3):
            call()
        torch.cuda.synchronize()
        t_iters = 20
        q0, q1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(s):
            torch.cuda._sleep(int(2e7))
            q0.record(s)
            for _ in range(t_iters):
                call()
            q1.record(s)
        torch.cuda.synchronize()
        t_ms = q0.elapsed_time(q1) / t_iters
        ng = (HIDDEN + 127) // 128
        tb = VOCAB * rb + VOCAB * ng * 2 + HIDDEN * 4 + VOCAB * 4
        trunk = {"workload": "kimi_linear_lm_head_q8g_163840x2304", "ms_per_call": t_ms,
                 "bytes_per_call": tb, "GBps": tb / (t_ms / 1e3) / 1e9,
                 "frac": tb / (t_ms / 1e3) / 1e9 / peaks()[0],
                 "l2": "383 MB per call, larger than L2"}
        del dW, ds

    # ---- config 4 (the K3-class layer, batches 1/16/64) at this N: layers
    # 101.., codebooks appended to layer 1's
    k3 = None
    if (world == 1 or ep_mode) and not args.decode_only and not args.no_k3:
        k3_res, k3_facts = k3_workload(args, rank, world, dev, dist, cb_books=base.books_raw,
                                       layer0=100)
        peak_k3 = peaks()[0]
        k3 = {"metric": K3_METRIC, "unit": UNIT, "batches": k3_res,
              "tok_per_s": {b: r["tok_per_s"] for b, r in k3_res.items()},
              "rank0_frac_of_hbm": {b: (r["rank0_GBps"] or 0) / peak_k3 for b, r in k3_res.items()},
              "config": dict(k3_facts, hidden=K3_HIDDEN, moe_inter=K3_INTER, top_k=K3_TOPK,
                             parallelism=f"ep{world}" if world > 1 else "single")}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(args.cpu_budget)
    engine = engine_slot_path(base) if world == 1 and not args.decode_only else None
    engine_step = None
    if rank == 0 and world == 1 and not args.decode_only and not args.no_engine_step:
        engine_step = engine_step_leg(args)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded; bf16-valued N(0,1) first h, N(0,0.02^2) codebooks, "
                    "uniform indices, random-init router/shared expert/norm weights)",
            "config": {"workload": "kimi_linear_48b_moe_decode", "hidden": HIDDEN,
                       "moe_inter": INTER, "experts": EXPERTS, "top_k": TOPK,
                       "shared_experts": 1, "moe_layers": nL,
                       "chained": "layer L+1's h is layer L's h_out (rmsnorm, MoE layer, "
                                  "residual add per layer)",
                       "global_batch": world,
                       "parallelism": (f"ep{world}" if ep_mode else f"replicas{world}")
                                      if world > 1 else "single",
                       "experts_per_gpu": count,
                       "l2": "inputs larger than L2 (~803 MB touched per step)",
                       "cuda_graphs": use_graphs},
            "gpu_launches": int(launches_per_step * args.steps),
            "clocks": ck,
            "e2e": e2e,
            "e2e_engine_slot": engine,
            "engine_step": engine_step,
            "roofline": {"bound": "hbm", "kernel": "gateup_kernel",
                         "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_source": peak_src,
                         "traffic": GATEUP_TRAFFIC_BYTES,
                         "bytes_per_launch": gateup_bytes(), "avg_launch_us": gu_avg * 1e3,
                         "layer_GBps": layer_bytes() / (ms_step / nL / 1e3) / 1e9,
                         "layer_frac": layer_bytes() / (ms_step / nL / 1e3) / 1e9 / peak},
            "kernels": kernels,
            "matvec": matvec,
            "prefill": prefill,
            "trunk_mvq": trunk,
            "parity": parity,
            "k3": k3,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    # Graphs that hold the library's NCCL calls must be gone before its
    # communicator is destroyed, or the teardown waits for good.
    torch.cuda.synchronize()
    graphs.clear()
    import gc
    gc.collect()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
        if ep_mode:
            ep.shutdown()
        dist.destroy_process_group()
    return 0


# ---------------------------------------------------------------- config 4

K3_HIDDEN, K3_INTER, K3_EXPERTS, K3_TOPK, K3_SHARED = 7168, 2048, 512, 16, 2048
K3_SCALE = 2.827
K3_LAYERS = 4                 # resident layers the steps cycle over
K3_BATCHES = (1, 16, 64)
K3_METRIC = "K3-class MoE layer tok/s (hidden 7168, 512 VQ3R experts, top-16)"


def k3_expert_bytes():
    from warp_b200 import synth
    idx = 2 * synth.index_bytes(K3_INTER, K3_HIDDEN, 3) + synth.index_bytes(K3_HIDDEN, K3_INTER, 3)
    return idx + 2 * (2 * K3_INTER + K3_HIDDEN)


def k3_trunk_bytes():
    ng_h, ng_s = (K3_HIDDEN + 127) // 128, (K3_SHARED + 127) // 128
    shared = (2 * K3_SHARED * ng_h * 128 + K3_HIDDEN * ng_s * 128
              + 2 * (2 * K3_SHARED * ng_h + K3_HIDDEN * ng_s))
    return K3_EXPERTS * K3_HIDDEN * 4, shared


def k3_cpu_sample(budget_s=10.0, threads=0):
    """The reference moe_layer at the K3-class matrix shapes on this host's
    cores: a 32-expert bank (top-16, so every token still runs 16 experts of
    7168 x 2048), bounded to about budget_s. Returns (s per token, cores,
    kind, sample)."""
    import oracle as O
    from warp_b200 import synth
    L = synth.moe_layer(SEED + 50, hidden=K3_HIDDEN, inter=K3_INTER, n_experts=32,
                        top_k=K3_TOPK, shared_inter=K3_SHARED, routed_scale=K3_SCALE)
    xs = synth.activations(SEED + 51, K3_HIDDEN, T=8)
    if O.ref_available():
        rm = O.RefMoe(L, max_tokens=1, threads=threads)
        run, kind, cores = rm.layer, "reference", O.ref().refh_pool_threads()
    else:
        rm, kind, cores = None, "port", 1
        run = lambda x: O.moe_layer(L, x)
    run(xs[0])
    t0 = time.perf_counter()
    run(xs[1])
    per = max(time.perf_counter() - t0, 1e-4)
    n = max(2, min(200, int(budget_s / per)))
    t0 = time.perf_counter()
    for i in range(n):
        run(xs[i % 8])
    dt = (time.perf_counter() - t0) / n
    if rm is not None:
        rm.close()
    return dt, cores, kind, (f"{n} single-token calls of the reference moe_layer at hidden "
                             f"7168 / inter 2048 / top-16 + shared expert, on a 32-expert bank "
                             f"(the per-token expert work of the 512-expert layer)")


def run_k3_reference(args):
    rank, world, _ = dist_setup(args.gpus)
    if rank != 0:
        return 0
    dt, cores, kind, sample = k3_cpu_sample(max(args.cpu_budget, 5.0))
    v = 1.0 / dt
    line = {"metric": K3_METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "impl": "reference",
            "config": {"workload": "k3_class_moe_layer_decode", "hidden": K3_HIDDEN,
                       "moe_inter": K3_INTER, "experts": K3_EXPERTS, "top_k": K3_TOPK,
                       "global_batch": 1, "parallelism": "cpu"},
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": cores, "kind": kind,
                             "sample": sample},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def k3_workload(args, rank, world, dev, dist, cb_books=None, layer0=0):
    """Config 4: one K3-class MoE layer per step, batches 1/16/64 tokens, on
    a device (and, with world > 1, an expert-parallel exchange) that is
    already set up. N = 1: the whole layer on one GPU (the batched layer
    call). N > 1: expert parallel, 512/N experts per rank; batch 1 is held
    by every rank (replicated trunk: routes agree, partial sums all-reduced
    through peer memory), larger batches are split B/N tokens per rank
    (tokens out to every rank, partial sums back to the tokens' ranks).
    Layers are numbered from layer0 + 1; cb_books, when given, are codebooks
    already loaded that the K3 books are appended to (the K3 records then
    name their own books after them). Returns the results and setup facts."""
    import torch
    import warp_b200 as wb
    from warp_b200 import synth
    ep = None
    if world > 1:
        from warp_b200 import ep
    E = args.k3_experts
    first, count = 0, E
    if world > 1:
        first, count = ep.ep_range(E, rank, world)
    nL = args.k3_layers
    books = synth.codebooks(np.random.default_rng(SEED + 20), 9)
    cb0 = 0
    if cb_books is not None:
        cb0 = cb_books.shape[0]
        books = np.concatenate([cb_books, books])
    wb.codebooks_load_f16(books)
    rb = synth.record_bytes(K3_INTER, K3_HIDDEN, 3)
    t_gen = time.perf_counter()
    chunk = 16
    for c0 in range(first, first + count, chunk):
        n = min(chunk, first + count - c0)
        recs = synth.bank_range(SEED + 30, 1, c0, n, cb0, K3_INTER, K3_HIDDEN)
        for L in range(1, nL + 1):
            synth.set_layer(recs, layer0 + L)
            wb.vq_bank_load(layer0 + L, E, rb, c0, n, recs.reshape(-1), K3_INTER, K3_HIDDEN, 3)
        del recs
    for L in range(1, nL + 1):
        router, sh = synth.trunk(SEED + 40 + L, K3_HIDDEN, E, K3_SHARED)
        wb.moe_trunk_load(layer0 + L, E, K3_HIDDEN, K3_TOPK, 1, K3_SCALE, router, None,
                          K3_SHARED, sh)
    t_gen = time.perf_counter() - t_gen
    s = torch.cuda.Stream(device=dev)
    ntok = 4
    results, graphs = {}, []
    expert_b = k3_expert_bytes()
    router_b, shared_b = k3_trunk_bytes()
    router_b = router_b * E // K3_EXPERTS
    for B in [int(b) for b in args.batches.split(",")]:
        if world > 1 and B > 1 and B % world:
            continue
        T = B if (world == 1 or B == 1) else B // world      # tokens this rank passes
        mode = "single" if world == 1 else ("rep" if B == 1 else "split")
        xs_h = synth.activations(SEED + 60 + B + (rank if mode == "split" else 0), K3_HIDDEN,
                                 T=ntok * nL * T).reshape(ntok, nL, T, K3_HIDDEN)
        xs = torch.from_numpy(xs_h).to(dev)
        out = torch.empty((nL, T, K3_HIDDEN), dtype=torch.float32, device=dev)
        # routes returned for the tokens this rank passed
        idx = torch.empty((ntok, nL, T, K3_TOPK), dtype=torch.int32, device=dev)
        w = torch.empty((ntok, nL, T, K3_TOPK), dtype=torch.float32, device=dev)

        def call(t, L):
            xp, op = xs[t, L].data_ptr(), out[L].data_ptr()
            ip, wp = idx[t, L].data_ptr(), w[t, L].data_ptr()
            if mode == "single":
                if T == 1:
                    wb.moe_layer_dev(layer0 + L + 1, xp, op, ip, wp, s.cuda_stream)
                else:
                    wb.moe_layer_part_dev(layer0 + L + 1, T, xp, op, 0, T, ip, wp, s.cuda_stream)
            elif mode == "rep":
                ep.moe_layer_rep_dev(layer0 + L + 1, T, xp, op, ip, wp, s.cuda_stream)
            else:
                ep.moe_layer_dev(layer0 + L + 1, T, xp, op, ip, wp, s.cuda_stream)

        def step_direct(t):
            for L in range(nL):
                call(t, L)

        with torch.cuda.stream(s):
            for t in range(ntok):
                step_direct(t)
        torch.cuda.synchronize()
        assert wb.device_errors() == 0
        # distinct experts each call reads on this rank, from the routes
        ih = idx.cpu().numpy()
        if mode == "split":           # every rank's tokens reach every rank
            allr = torch.from_numpy(ih).to(dev)
            gath = [torch.empty_like(allr) for _ in range(world)]
            dist.all_gather(gath, allr)
            ih = np.concatenate([g.cpu().numpy() for g in gath], axis=2)
        local_e = [np.unique(ih[t, L][(ih[t, L] >= first) & (ih[t, L] < first + count)]).size
                   for t in range(ntok) for L in range(nL)]
        ex_rank = float(np.mean(local_e))
        # per-rank algorithmic bytes of one layer call: local experts, the
        # replicated router, the shared expert for this rank's share of the
        # tokens (rounded up: one token's share is a whole read), the tokens
        sh_tokens = T if mode != "rep" else (rank + 1) * T // world - rank * T // world
        call_bytes = (ex_rank * expert_b + router_b + (shared_b if sh_tokens else 0)
                      + 2 * T * K3_HIDDEN * 4)
        gs = []
        try:
            for t in range(ntok):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=s, capture_error_mode="thread_local"):
                    step_direct(t)
                gs.append(g)
            graphs.extend(gs)
            use_graphs = True
        except Exception as e:
            print(f"graph capture unavailable: {e}", file=sys.stderr)
            gs, use_graphs = [], False

        def step(k):
            if use_graphs:
                gs[k % ntok].replay()
            else:
                step_direct(k % ntok)

        reps = max(1, args.steps // nL)
        with torch.cuda.stream(s):
            for k in range(max(args.warmup, 3)):
                step(k)
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        with torch.cuda.stream(s):
            for k in range(reps):
                step(k)
        e1.record(s)
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        ms = e0.elapsed_time(e1)
        my_ms = ms
        if dist:
            tt = torch.tensor([ms], dtype=torch.float64, device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            ms = float(tt.item())
        calls = reps * nL
        ms_call = ms / calls
        per_rank_GBps = call_bytes / (my_ms / calls / 1e3) / 1e9
        # per-kernel device times: one step's launches queued behind a
        # GPU-side sleep, so each event pair brackets kernel time only
        wb.profile(True)
        with torch.cuda.stream(s):
            torch.cuda._sleep(int(2e7))
            step_direct(0)
        torch.cuda.synchronize()
        ph = wb.profile_read()
        wb.profile(False)
        if dist:
            dist.barrier()
        results[B] = {"tokens_per_call": B, "tokens_per_rank": T, "mode": mode,
                      "ms_per_layer_call": ms_call, "tok_per_s": B / (ms_call / 1e3),
                      "local_experts_per_call": ex_rank,
                      "rank0_bytes_per_call": None, "rank0_GBps": None,
                      "rank0_kernel_us_per_call": {k: v[0] * 1e3 / nL for k, v in ph.items()
                                                   if v[1]}}
        # rank 0's own figures (bytes and GB/s over its own time)
        if rank == 0:
            results[B]["rank0_bytes_per_call"] = call_bytes
            results[B]["rank0_GBps"] = per_rank_GBps
        assert wb.device_errors() == 0
    torch.cuda.synchronize()
    graphs.clear()
    import gc
    gc.collect()
    torch.cuda.synchronize()
    return results, {"experts": E, "experts_per_gpu": count, "resident_layers": nL,
                     "setup_s": t_gen}


def run_k3(args):
    """Config 4 on its own (--workload k3): the K3-class layer at batches
    1/16/64 over N GPUs (k3_workload)."""
    import torch
    import warp_b200 as wb

    rank, world, local = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=dev)
    wb.init(local)
    if world > 1:
        from warp_b200 import ep
        ep.setup(rank, world)
    clocks = Clocks(local)
    clocks.start()
    results, facts = k3_workload(args, rank, world, dev, dist)
    ck = clocks.stop()
    peak, peak_src = peaks()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        dt, cores, kind, sample = k3_cpu_sample(args.cpu_budget)
        cpu = {"value": 1.0 / dt, "unit": UNIT, "cores": cores, "kind": kind, "sample": sample}
    if rank == 0:
        head = results[max(results)]
        line = {
            "metric": K3_METRIC, "value": head["tok_per_s"], "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": head["ms_per_layer_call"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded per expert; uniform indices, N(0,0.02^2) codebooks, "
                    "router rows N(0,1/hidden), bf16-valued N(0,1) tokens)",
            "config": {"workload": "k3_class_moe_layer_decode", "hidden": K3_HIDDEN,
                       "moe_inter": K3_INTER, "experts": facts["experts"], "top_k": K3_TOPK,
                       "shared_experts": 1, "resident_layers": facts["resident_layers"],
                       "global_batch": max(results), "experts_per_gpu": facts["experts_per_gpu"],
                       "parallelism": f"ep{world}" if world > 1 else "single",
                       "l2": f"steps cycle over {facts['resident_layers']} resident layers and 4 "
                             "token slots (> 126 MB of distinct weights between repeats at the "
                             "default 4 layers x 512 experts)",
                       "cuda_graphs": True, "setup_s": facts["setup_s"]},
            "batches": results,
            "roofline": {"bound": "hbm", "peak": peak, "peak_source": peak_src,
                         "unit": "GB/s",
                         "rank0_frac_by_batch": {b: (r["rank0_GBps"] or 0) / peak
                                                 for b, r in results.items()}},
            "clocks": ck,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        ep.shutdown()
        dist.destroy_process_group()
    return 0


# ---------------------------------------------------------------- config 5

ENGINE_RUN = os.path.join(ROOT, "integration", "_build", "engine_run")
CUDA_ENGINE = os.path.join(ROOT, "integration", "_build", "libwaste_engine_cuda.so")
REF_ENGINE = os.path.join(ROOT, "oracle", "_ref", "libwaste_ref.so")
C5_PROMPT = [1, 17, 4242, 99, 12345, 7, 808, 3]


def _engine(lib, cdir, steps, env=None, timeout=3600):
    """Runs integration/_build/engine_run: per eval (ms, next token), the
    logits, open time and the backend's launch count."""
    out = tempfile.mktemp(suffix=".bin")
    r = subprocess.run([ENGINE_RUN, lib, cdir, out, str(steps)] + [str(t) for t in C5_PROMPT],
                       capture_output=True, text=True, timeout=timeout,
                       env=dict(os.environ, **(env or {})))
    if r.returncode != 0:
        raise RuntimeError(f"engine_run failed: {r.stdout[-2000:]} {r.stderr[-2000:]}")
    res = {"ms": [], "tok": [], "launches": None, "open_ms": None, "build": ""}
    for line in r.stdout.splitlines():
        if line.startswith("build:"):
            res["build"] = line[7:]
        elif line.startswith("open:"):
            res["open_ms"] = float(line.split()[1])
        elif line.startswith("eval "):
            res["tok"].append(int(line.split("next token ")[1].split()[0]))
            res["ms"].append(float(line.split("(")[1].split()[0]))
        elif line.startswith("cuda launches:"):
            res["launches"] = int(line.split(":")[1])
    raw = np.fromfile(out, dtype=np.int32)
    os.unlink(out)
    nev, vocab = int(raw[0]), int(raw[1])
    res["logits"] = raw[2:].reshape(nev, 1 + vocab)[:, 1:].copy().view(np.float32)
    return res


def _container(args):
    from warp_b200 import synth
    import shutil
    cdir = args.container
    if not cdir:                     # the first place with room for ~19 GB (tmpfs first)
        for base in ("/dev/shm", tempfile.gettempdir(), ROOT):
            try:
                if os.access(base, os.W_OK) and shutil.disk_usage(base).free > (24 << 30):
                    cdir = os.path.join(base, "warp_c5")
                    break
            except OSError:
                continue
        if not cdir:
            raise SystemExit("no file system with 24 GB free for the config-5 container")
    t0 = time.time()
    if not os.path.exists(os.path.join(cdir, "manifest.json")):
        synth.write_container(cdir, seed=SEED)
    return cdir, time.time() - t0


def run_engine_reference(args):
    """The unmodified reference engine on config 5's container (CPU)."""
    cdir, wt = _container(args)
    steps = max(3, min(args.steps, 8))
    ref = _engine(REF_ENGINE, cdir, args.warmup + steps)
    dec = ref["ms"][1 + args.warmup:]
    v = 1e3 / statistics.mean(dec)
    print(json.dumps({"impl": "reference", "metric": ENGINE_METRIC, "value": v, "unit": UNIT,
                      "n_gpus": 1, "steps": len(dec), "warmup": args.warmup,
                      "ms_per_step": statistics.mean(dec), "higher_is_better": True,
                      "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                      "data": "synthetic (seeded container)",
                      "config": {"workload": "kimi_linear_48b_full_decode_step", "layers": 27},
                      "cpu_baseline": {"value": v, "unit": UNIT, "cores": os.cpu_count(),
                                       "kind": "reference",
                                       "sample": f"{len(dec)} decode steps through waste_eval"},
                      "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0,
                              "d2h_bytes_per_step": 0}}), flush=True)
    return 0


ENGINE_METRIC = ("decode tok/s through the engine's waste.h (full Kimi-Linear-48B-shaped decode "
                 "step: 27 layers, KDA + MLA attention, 26 VQ3R MoE layers, batch 1)")


def engine_step_measure(args, steps=10, warmup=3):
    """Config 5 measured: the patched engine's decode steps on the synthetic
    container (clocks sampled meanwhile), then a bounded sample of the
    unmodified engine on it, and their agreement."""
    def rel_l2(a, b):
        a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
        return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
    cdir, wt = _container(args)
    clk = Clocks(0)
    clk.start()
    cu = _engine(CUDA_ENGINE, cdir, warmup + steps)
    clocks = clk.stop()
    dec = cu["ms"][1 + warmup:]
    rs = max(3, min(steps, 8))
    ref = _engine(REF_ENGINE, cdir, warmup + rs)
    rdec = ref["ms"][1 + warmup:]
    m = min(len(cu["tok"]), len(ref["tok"]))
    return {"cu": cu, "dec": dec, "ref": ref, "rdec": rdec, "clocks": clocks, "write_s": wt,
            "tokens_equal": cu["tok"][:m] == ref["tok"][:m], "evals_compared": m,
            "worst": max(rel_l2(cu["logits"][e], ref["logits"][e]) for e in range(m))}


def engine_step_leg(args):
    """The default line's config-5 object (one GPU), or None when the engine
    builds are missing."""
    if not (os.path.exists(ENGINE_RUN) and os.path.exists(CUDA_ENGINE) and
            os.path.exists(REF_ENGINE)):
        return None
    r = engine_step_measure(args)
    v = 1e3 / statistics.mean(r["dec"])
    cpu = 1e3 / statistics.mean(r["rdec"])
    return {"metric": ENGINE_METRIC, "value": v, "unit": UNIT, "steps": len(r["dec"]),
            "ms_per_step": statistics.mean(r["dec"]),
            "timing": "wall clock of each decode step's waste_eval (host API, copies included)",
            "config": {"workload": "kimi_linear_48b_full_decode_step", "layers": 27,
                       "kda_layers": 21, "mla_layers": 6, "moe_layers": 26,
                       "container_write_s": r["write_s"], "engine_open_ms": r["cu"]["open_ms"]},
            "clocks": r["clocks"],
            "parity": {"tokens_equal": r["tokens_equal"], "worst_logits_rel_l2": r["worst"],
                       "evals_compared": r["evals_compared"]},
            "cpu_baseline": {"value": cpu, "unit": UNIT, "cores": os.cpu_count(),
                             "kind": "reference",
                             "sample": f"{len(r['rdec'])} decode steps of the unmodified engine"}}


def run_engine_workload(args):
    r = engine_step_measure(args, steps=args.steps, warmup=args.warmup)
    cu, dec = r["cu"], r["dec"]
    v = 1e3 / statistics.mean(dec)
    cpu = 1e3 / statistics.mean(r["rdec"])
    launches = cu["launches"] or 0
    per_step = launches / max(len(cu["ms"]), 1)
    hid, vocab = 2304, 163840
    line = {"metric": ENGINE_METRIC, "value": v, "unit": UNIT, "n_gpus": 1, "steps": len(dec),
            "warmup": args.warmup, "ms_per_step": statistics.mean(dec),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded Kimi-Linear-48B-shaped container written by "
                    "warp_b200.synth: random trunk in its Q8G/Q4G/F32 formats, N(0, 0.02^2) "
                    "codebooks, uniform expert indices)",
            "config": {"workload": "kimi_linear_48b_full_decode_step", "layers": 27,
                       "kda_layers": 21, "mla_layers": 6, "moe_layers": 26, "experts": 256,
                       "top_k": 8, "hidden": hid, "vocab": vocab, "prompt_tokens": len(C5_PROMPT),
                       "timing": "wall clock of each decode step's waste_eval (host API)",
                       "container_write_s": r["write_s"], "engine_open_ms": cu["open_ms"],
                       "backend": cu["build"]},
            "gpu_launches": int(per_step * len(dec)), "clocks": r["clocks"],
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": hid * 4,
                    "d2h_bytes_per_step": vocab * 4},
            "parity": {"tokens_equal": r["tokens_equal"], "worst_logits_rel_l2": r["worst"],
                       "evals_compared": r["evals_compared"],
                       "against": "the unmodified reference engine, same container and prompt"},
            "cpu_baseline": {"value": cpu, "unit": UNIT, "cores": os.cpu_count(),
                             "kind": "reference",
                             "sample": f"{len(r['rdec'])} decode steps of the unmodified engine "
                                       "through waste_eval on the same container"}}
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("warp", "reference"), default="warp")
    ap.add_argument("--layers", type=int, default=MOE_LAYERS)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true", help="skip the oracle check")
    ap.add_argument("--no-k3", action="store_true",
                    help="skip the config-4 (K3-class) leg of the default workload")
    ap.add_argument("--decode-only", action="store_true",
                    help="only the decode chain (no matvec, prefill or engine-slot legs): "
                         "for profiling runs")
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    ap.add_argument("--parallel", choices=("ep", "replicas"), default="ep",
                    help="with --gpus N > 1: expert parallel (default) or N replicas")
    ap.add_argument("--workload", choices=("kimi", "k3", "engine"), default="kimi",
                    help="kimi: the Kimi-Linear decode step (default); k3: one K3-class "
                         "MoE layer at batches 1/16/64; engine: config 5 through waste.h")
    ap.add_argument("--no-engine-step", action="store_true",
                    help="skip the config-5 leg (the whole decode step through the engine)")
    ap.add_argument("--container", default=None,
                    help="engine: where the synthetic container is (written if missing)")
    ap.add_argument("--batches", default="1,16,64", help="k3: global batches")
    ap.add_argument("--k3-experts", type=int, default=K3_EXPERTS,
                    help="k3: experts per layer (fewer only for small profiling cases)")
    ap.add_argument("--k3-layers", type=int, default=K3_LAYERS, help="k3: resident layers")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.workload == "k3":
        return run_k3_reference(args) if args.impl == "reference" else run_k3(args)
    if args.workload == "engine":
        if args.gpus != 1:
            raise SystemExit("--workload engine runs one engine process on one GPU")
        if args.impl == "reference":
            return run_engine_reference(args)
        return run_engine_workload(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_warp(args)


if __name__ == "__main__":
    sys.exit(main())
