"""One kernel of the library at a stated size, for timing and for an ncu
capture of that kernel alone.

    python -m warp_b200.profile_cases <case> [--reps N]

Cases (synthetic, seeded data; every input larger than L2 unless said):
  vq4p     32 VQ4P matvecs of 4096 x 4096 (four 64-entry stages, 6-bit
           indices packed four to three bytes) in one call: 201 MB of indices
  lm_head  the trunk matvec (mvq_rows_f32) at the Kimi-Linear lm_head shape,
           163840 x 2304 Q8G: 383 MB per call
  kda      the KDA decode step at the Kimi-Linear shape (32 heads, K = V =
           128), cycling over 80 layers' recurrent states (2 MB each, 168 MB)
  encode   the converter's RVQ encoder: 4M 8-dim vectors, three stages of
           256 entries (128 MB in, 12 MB of codes out)

Prints the average time of a launch (CUDA events around `reps` calls after
three untimed ones) and the algorithmic bytes a call moves.
"""
from __future__ import annotations

import argparse
import json
import sys

import numpy as np


def _events(torch, stream, fn, reps):
    for _ in range(3):
        fn(0)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        torch.cuda._sleep(int(5e7))          # host enqueue runs ahead of the device
        e0.record(stream)
        for k in range(reps):
            fn(k)
        e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def main(argv=None):
    import torch
    import warp_b200 as wb
    from warp_b200 import synth

    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=("vq4p", "lm_head", "kda", "encode"))
    ap.add_argument("--reps", type=int, default=20)
    args = ap.parse_args(argv)
    wb.init(0)
    dev = torch.device("cuda", 0)
    s = torch.cuda.Stream(device=dev)
    rng = np.random.default_rng(4242)
    out = {"case": args.case}
    if args.case == "vq4p":
        G, M, N = 32, 4096, 4096
        wb.codebooks_load_f16(synth.codebooks(rng, 4, entries=synth.ENTRIES_VQ4P))
        mats = [synth.random_matrix(rng, M, N, stages=4) for _ in range(G)]
        d_idx = torch.from_numpy(np.stack([m[0] for m in mats])).to(dev)
        d_sc = torch.from_numpy(np.stack([m[1].view(np.int16) for m in mats])).to(dev)
        d_x = torch.from_numpy(synth.activations(7, N, T=G)).to(dev)
        d_y = torch.empty((G, M), dtype=torch.float32, device=dev)
        p = ([d_idx[g].data_ptr() for g in range(G)], [d_sc[g].data_ptr() for g in range(G)],
             [d_x[g].data_ptr() for g in range(G)], [d_y[g].data_ptr() for g in range(G)])
        ms = _events(torch, s, lambda k: wb.vq4p_matvec_dev(*p, M, N, 0, s.cuda_stream), args.reps)
        nbytes = G * (synth.index_bytes(M, N, 4) + 2 * M + 4 * N + 4 * M) + 4 * 64 * 8 * 4
    elif args.case == "lm_head":
        V, H = 163840, 2304
        raw, sc, rb = synth.trunk_tensor(rng, V, H, 8)
        dW = torch.from_numpy(raw).to(dev)
        ds = torch.from_numpy(sc.view(np.int16)).to(dev)
        dx = torch.from_numpy(synth.activations(13, H)[0]).to(dev)
        dy = torch.empty((V,), dtype=torch.float32, device=dev)
        ms = _events(torch, s, lambda k: wb.mvq_rows_dev(dy.data_ptr(), dW.data_ptr(), ds.data_ptr(),
                                                          dx.data_ptr(), 0, V, H, 128, 8, rb,
                                                          s.cuda_stream), args.reps)
        nbytes = raw.nbytes + sc.nbytes + H * 4 + V * 4
    elif args.case == "kda":
        H, K, V, L = 32, 128, 128, 80
        dS = torch.zeros((L, H, K, V), dtype=torch.float32, device=dev)
        q, k, v = (torch.randn(H * K, device=dev) for _ in range(3))
        g = -torch.rand(H * K, device=dev)
        beta = torch.rand(H, device=dev)
        do = torch.empty(H * V, device=dev)
        ms = _events(torch, s, lambda j: wb.kda_step_dev(H, K, V, q.data_ptr(), k.data_ptr(),
                                                          v.data_ptr(), g.data_ptr(),
                                                          beta.data_ptr(), dS[j % L].data_ptr(),
                                                          do.data_ptr(), s.cuda_stream),
                     args.reps)
        nbytes = 2 * H * K * V * 4 + 3 * H * K * 4 + H * 4 + H * V * 4   # state read + write
    else:
        n, dim, stages = 4 << 20, 8, 3
        # the converter's inputs: rows of W / scale (|x| <= 1), books shrinking by stage
        books = np.stack([rng.normal(0.0, 0.3 / (k + 1), (256, dim)) for k in range(stages)]
                         ).astype(np.float32)
        dX = torch.from_numpy(np.clip(rng.normal(0.0, 0.4, (n, dim)), -1, 1).astype(np.float32)
                              ).to(dev)
        dB = torch.from_numpy(np.ascontiguousarray(books)).to(dev)
        dO = torch.empty((n, stages), dtype=torch.uint8, device=dev)
        ms = _events(torch, s, lambda k: wb.vq_encode_dev(dX.data_ptr(), n, dB.data_ptr(), stages,
                                                           256, dim, dO.data_ptr(), s.cuda_stream),
                     args.reps)
        nbytes = n * dim * 4 + n * stages + books.nbytes
        out["flop_per_call"] = 3 * n * stages * 256 * dim
    out.update(ms_per_call=ms, bytes_per_call=int(nbytes), GBps=nbytes / (ms / 1e3) / 1e9,
               device_errors=wb.device_errors())
    print(json.dumps(out))
    return 0


if __name__ == "__main__":
    sys.exit(main())
