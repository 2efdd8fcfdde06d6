"""One rank of the two-GPU expert-parallel test (launched by
tests/test_ep_gpu.py under torchrun): each rank holds half of the experts
of two layers, decodes its own tokens (and tokens every rank holds)
through the peer-memory exchange and then the NCCL one, and checks them
against the oracle on the whole layer."""
import datetime
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))

import numpy as np
import torch
import torch.distributed as dist

import oracle as O
import warp_b200 as wb
from golden_cases import rel_l2
from warp_b200 import ep, synth

TOL = 2e-5


def skipped_call(rank, world, L, dev):
    """A rank that does not make its layer call. With a short peer-wait
    limit, rank 0's call gives up on rank 1's flags and reports
    DERR_PEER_WAIT instead of hanging, and the device stays usable. Both
    ranks first make one call together: the first call builds the
    mailboxes, which takes a collective. After the skipped call, both
    ranks' next call fails (refused, or PEER_WAIT) until the exchange is
    built again."""
    os.environ["WASTE_CUDA_EP_WAIT_POLLS"] = str(1 << 20)
    ep.setup(rank, world)
    x = synth.activations(500, L.hidden, T=1)
    dx = torch.from_numpy(x).to(dev)
    out = torch.empty((1, L.hidden), device=dev)
    dist.barrier()
    ep.moe_layer_rep_dev(L.layer, 1, dx.data_ptr(), out.data_ptr())
    torch.cuda.synchronize()
    assert wb.device_errors() == 0, "the joint call"
    dist.barrier()
    if rank == 0:                            # rank 1 sits this one out
        ep.moe_layer_rep_dev(L.layer, 1, dx.data_ptr(), out.data_ptr())
        torch.cuda.synchronize()
        errs = wb.device_errors()
        assert errs & wb.DERR_PEER_WAIT, errs
        assert wb.device_errors() == 0       # reading cleared the bits
    dist.barrier()
    # The ranks' epochs are now out of step. One more joint call: rank 0,
    # which saw the bit, is refused on the host; rank 1 launches, and its
    # waits fail at once on the poison word rank 0 left in its mailbox.
    # Neither returns outputs as if they were valid.
    if rank == 0:
        try:
            ep.moe_layer_rep_dev(L.layer, 1, dx.data_ptr(), out.data_ptr())
            raise AssertionError("rank 0's call after a peer wait was not refused")
        except wb.WasteCudaError as e:
            assert e.rc == wb.E_DEVICE, e
    else:
        ep.moe_layer_rep_dev(L.layer, 1, dx.data_ptr(), out.data_ptr())
        torch.cuda.synchronize()
        errs = wb.device_errors()
        assert errs & wb.DERR_PEER_WAIT, errs
        try:                                  # and now the host refuses too
            ep.moe_layer_rep_dev(L.layer, 1, dx.data_ptr(), out.data_ptr())
            raise AssertionError("rank 1's call after a peer wait was not refused")
        except wb.WasteCudaError as e:
            assert e.rc == wb.E_DEVICE, e
    dist.barrier()
    ep.shutdown()
    del os.environ["WASTE_CUDA_EP_WAIT_POLLS"]


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    wb.init(local)
    ep.setup(rank, world)
    layers = [synth.moe_layer(71 + k, hidden=768, inter=384, n_experts=64, top_k=8,
                              shared_inter=384, layer=50 + k, with_bias=bool(k), cb_base=9 * k)
              for k in range(2)]
    first, count = ep.ep_range(64, rank, world)
    wb.codebooks_load_f16(np.concatenate([layers[0].books_raw[:9], layers[1].books_raw[9:18]]))
    for L in layers:
        wb.vq_bank_load(L.layer, L.n_experts, L.rec_bytes, first, count,
                        L.bank[first * L.rec_bytes:], L.inter, L.hidden, L.stages)
        wb.moe_trunk_load(L.layer, L.n_experts, L.hidden, L.top_k, L.renorm, L.routed_scale,
                          L.router, L.bias, L.shared_inter, L.sh)
        wb.moe_norm_load(L.layer, synth.norm_weight(80 + L.layer, L.hidden), synth.NORM_EPS)
    T = 3
    dev = torch.device("cuda", local)

    def check(mode):
        for rep in range(2):                 # twice: the exchange's flags only grow
            for L in layers:
                x = synth.activations(100 + 10 * rank + L.layer + rep, L.hidden, T=T)
                dx = torch.from_numpy(x).to(dev)
                out = torch.empty((T, L.hidden), device=dev)
                idx = torch.empty((T, L.top_k), dtype=torch.int32, device=dev)
                ep.moe_layer_dev(L.layer, T, dx.data_ptr(), out.data_ptr(), idx.data_ptr())
                torch.cuda.synchronize()
                out, idx = out.cpu().numpy(), idx.cpu().numpy()
                for t in range(T):
                    ro, ri, _ = O.moe_layer(L, x[t], fma=1)
                    assert np.array_equal(idx[t], ri), (mode, rank, L.layer, t)
                    r = rel_l2(out[t], ro)
                    assert r < TOL, (mode, rank, L.layer, t, r)
                # the same layer for tokens every rank holds (a batch of one;
                # nine: the decode-sized forms over several tokens; 25: the
                # batched forms — many-token router, gate/up tiles that take
                # a token's local experts in rounds, the separate SiLU
                # kernel), interleaved with the calls above
                for Tr in (1, 9, 25):
                    xr = synth.activations(300 + L.layer + rep + Tr, L.hidden, T=Tr)
                    dx = torch.from_numpy(xr).to(dev)
                    out = torch.empty((Tr, L.hidden), device=dev)
                    idx = torch.empty((Tr, L.top_k), dtype=torch.int32, device=dev)
                    ep.moe_layer_rep_dev(L.layer, Tr, dx.data_ptr(), out.data_ptr(),
                                         idx.data_ptr())
                    torch.cuda.synchronize()
                    out, idx = out.cpu().numpy(), idx.cpu().numpy()
                    for t in range(Tr):
                        ro, ri, _ = O.moe_layer(L, xr[t], fma=1)
                        assert np.array_equal(idx[t], ri), (mode, "rep", rank, L.layer, t)
                        r = rel_l2(out[t], ro)
                        assert r < TOL, (mode, "rep", rank, L.layer, t, r)
        # the MoE block (rmsnorm, layer, residual) chained over both layers,
        # split and replicated
        for rep_mode in (False, True):
            h0 = synth.activations(400 + rank * (not rep_mode) + 7 * rep_mode, 768, T=T)
            h = torch.from_numpy(h0.copy()).to(dev)
            hn = torch.empty_like(h)
            ref = h0.copy()
            for L in layers:
                call = ep.moe_block_rep_dev if rep_mode else ep.moe_block_dev
                call(L.layer, T, h.data_ptr(), hn.data_ptr())
                torch.cuda.synchronize()
                got = hn.cpu().numpy()
                hin = h.cpu().numpy()
                for t in range(T):
                    ro, _, _ = O.moe_block(L, hin[t], synth.norm_weight(80 + L.layer, 768),
                                           synth.NORM_EPS)
                    r = rel_l2(got[t] - hin[t], ro - hin[t])
                    assert r < TOL, (mode, "block", rep_mode, rank, L.layer, t, r)
                    ref[t], _, _ = O.moe_block(L, ref[t], synth.norm_weight(80 + L.layer, 768),
                                               synth.NORM_EPS)
                h, hn = hn, h
            fin = h.cpu().numpy()
            for t in range(T):
                assert rel_l2(fin[t], ref[t]) < TOL, (mode, "block chain", rep_mode, rank, t)
        assert wb.device_errors() == 0, mode

    check("peer memory")                     # the default exchange
    dist.barrier()
    ep.shutdown()
    skipped_call(rank, world, layers[0], dev)
    os.environ["WASTE_CUDA_EP_P2P"] = "0"    # the NCCL exchange, same banks
    ep.setup(rank, world)
    check("nccl")
    dist.barrier()
    ep.shutdown()
    dist.destroy_process_group()
    print(f"ep_worker ok rank {rank}", flush=True)


if __name__ == "__main__":
    main()
