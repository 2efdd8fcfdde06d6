"""Expert parallelism's host logic on CPU: two gloo ranks (no GPU).

What the device path relies on, checked with the oracle standing in for the
kernels:
  * the library's split gives every expert to exactly one rank;
  * rank 0's NCCL unique id reaches every rank unchanged (warp_b200.ep);
  * the per-rank partial sums (each rank's own experts, in router order) add
    up over the ranks to the routed part of the layer, within 2e-5, both for
    a batch split over the ranks and for one every rank holds.
"""
import os
import socket

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TOL = 2e-5


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def partial_reference(L, x, first, count):
    """One rank's share of the routed sum, from the oracle: per token, the
    routed experts in [first, first+count), in router order, weighted."""
    import oracle as O
    out = np.zeros((x.shape[0], L.hidden), dtype=np.float32)
    for t in range(x.shape[0]):
        _, idx, w = O.moe_layer(L, x[t], fma=1)
        mine = [(int(e), float(wj)) for e, wj in zip(idx, w) if first <= e < first + count]
        if mine:
            out[t] = O.moe_experts(L, np.array([e for e, _ in mine], np.int32),
                                   np.array([wj for _, wj in mine], np.float32), x[t], fma=1)
    return out


def _worker(rank, world, port, q):
    import sys
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import datetime

    import torch
    import torch.distributed as dist

    import oracle as O
    from warp_b200 import ep, synth
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=60))
        # 1. the split
        E = 24
        first, count = ep.ep_range(E, rank, world)
        owned = torch.zeros(E, dtype=torch.int32)
        owned[first:first + count] = 1
        dist.all_reduce(owned)
        assert owned.tolist() == [1] * E, owned.tolist()
        # 2. the id
        uid = ep.unique_id() if rank == 0 else None
        got = ep.share_id(uid, rank)
        ids = [None] * world
        dist.all_gather_object(ids, got)
        assert len(got) == ep.ID_BYTES and all(i == ids[0] for i in ids)
        if rank == 0:
            assert got == uid
        # 3. partial sums over the ranks' experts add up to the routed part
        L = synth.moe_layer(41, hidden=128, inter=64, n_experts=E, top_k=6, shared_inter=64,
                            layer=3)
        # (a batch split over the ranks: every rank's tokens go to every
        # rank, each computes its experts for all of them, and a rank's own
        # rows of the summed partials are its tokens' routed outputs)
        T = 3
        x = synth.activations(42 + rank, L.hidden, T=T)       # this rank's tokens
        xs = [torch.zeros((T, L.hidden)) for _ in range(world)]
        dist.all_gather(xs, torch.from_numpy(x))
        x_all = torch.cat(xs).numpy()
        part = torch.from_numpy(partial_reference(L, x_all, first, count))
        dist.all_reduce(part)
        mine = part[rank * T:(rank + 1) * T].numpy()
        for t in range(T):
            _, idx, w = O.moe_layer(L, x[t], fma=1)
            full = O.moe_experts(L, idx, w, x[t], fma=1)
            rel = float(np.linalg.norm(mine[t] - full) / np.linalg.norm(full))
            assert rel < TOL, rel
        # 4. a batch every rank holds (the replicated-token call): each rank
        # its own experts for all tokens, the sum over ranks is every
        # token's routed output on every rank
        xr = synth.activations(43, L.hidden, T=2)             # the same seed everywhere
        rp = torch.from_numpy(partial_reference(L, xr, first, count))
        dist.all_reduce(rp)
        for t in range(xr.shape[0]):
            _, idx, w = O.moe_layer(L, xr[t], fma=1)
            full = O.moe_experts(L, idx, w, xr[t], fma=1)
            rel = float(np.linalg.norm(rp[t].numpy() - full) / np.linalg.norm(full))
            assert rel < TOL, rel
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:  # reported to the parent
        q.put((rank, f"{type(e).__name__}: {e}"))


def test_expert_parallel_host_logic_gloo():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port, world = _free_port(), 2
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            r, msg = q.get(timeout=240)
            res[r] = msg
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert res == {r: "ok" for r in range(world)}, res


def test_ep_range_covers_experts():
    from warp_b200 import ep
    for E in (1, 7, 256, 512):
        for world in (1, 2, 3, 8):
            if world > E:
                continue
            spans = [ep.ep_range(E, r, world) for r in range(world)]
            assert spans[0][0] == 0
            for (f0, c0), (f1, _) in zip(spans, spans[1:]):
                assert f0 + c0 == f1
            assert spans[-1][0] + spans[-1][1] == E
            assert max(c for _, c in spans) - min(c for _, c in spans) <= 1
    with pytest.raises(Exception):
        ep.ep_range(8, 2, 2)
