"""Expert parallelism for the MoE layer: one process per GPU, the experts of
every layer split into contiguous ranges over the ranks, the trunk (router,
bias, shared expert) replicated, and the routed tokens exchanged with NCCL
over NVLink inside the library (include/waste_cuda.h, waste_cuda_ep_*).

This module is the host-side set-up: rank 0 makes the NCCL unique id, the id
travels to every rank over an existing torch.distributed group (gloo or
NCCL; a C engine would use any channel it has), and every rank joins the
library's communicator. The per-layer call is plain C.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _check, load_library

ID_BYTES = 128          # sizeof(ncclUniqueId)


def ep_range(n_experts: int, rank: int, world: int) -> tuple[int, int]:
    """(first, count): rank's contiguous share of n_experts (the library's
    own split, [rank*n/world, (rank+1)*n/world))."""
    f, c = C.c_int(), C.c_int()
    _check(load_library().waste_cuda_ep_range(n_experts, rank, world, C.byref(f), C.byref(c)))
    return f.value, c.value


def unique_id() -> bytes:
    buf = (C.c_ubyte * ID_BYTES)()
    _check(load_library().waste_cuda_ep_unique_id(buf, ID_BYTES))
    return bytes(buf)


def share_id(uid: bytes | None, rank: int, group=None) -> bytes:
    """Rank 0's id on every rank, through torch.distributed (CPU tensor for
    gloo; the group's device otherwise)."""
    import torch
    import torch.distributed as dist
    backend = dist.get_backend(group)
    dev = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else "cpu"
    t = torch.zeros(ID_BYTES, dtype=torch.uint8, device=dev)
    if rank == 0:
        t.copy_(torch.frombuffer(bytearray(uid), dtype=torch.uint8))
    dist.broadcast(t, src=0, group=group)
    return bytes(t.cpu().numpy().tobytes())


def init(rank: int, world: int, uid: bytes):
    """Joins the library's communicator (blocks until every rank has)."""
    b = (C.c_ubyte * ID_BYTES).from_buffer_copy(uid)
    _check(load_library().waste_cuda_ep_init(rank, world, b, ID_BYTES))


def setup(rank: int, world: int, group=None):
    """unique_id on rank 0, shared over `group`, then init on every rank."""
    uid = unique_id() if rank == 0 else None
    init(rank, world, share_id(uid, rank, group))


def shutdown():
    load_library().waste_cuda_ep_shutdown()


def moe_layer_dev(layer: int, T: int, d_x: int, d_out: int, d_idx: int = 0, d_w: int = 0,
                  stream: int = 0):
    """This rank's T tokens through the expert-parallel layer (device
    pointers; the same T on every rank)."""
    v = lambda p: C.c_void_p(int(p) or None)
    _check(load_library().waste_cuda_ep_moe_layer_dev(layer, T, v(d_x), v(d_out), v(d_idx),
                                                      v(d_w), v(stream)))


def moe_layer_rep_dev(layer: int, T: int, d_x: int, d_out: int, d_idx: int = 0, d_w: int = 0,
                      stream: int = 0):
    """T tokens that every rank holds (the same on every rank) through the
    expert-parallel layer; every rank receives all T outputs."""
    v = lambda p: C.c_void_p(int(p) or None)
    _check(load_library().waste_cuda_ep_moe_layer_rep_dev(layer, T, v(d_x), v(d_out),
                                                          v(d_idx), v(d_w), v(stream)))


def moe_block_dev(layer: int, T: int, d_h: int, d_out: int, d_idx: int = 0, d_w: int = 0,
                  stream: int = 0):
    """This rank's T tokens through the expert-parallel MoE block:
    h + moe_layer(rmsnorm(h))."""
    v = lambda p: C.c_void_p(int(p) or None)
    _check(load_library().waste_cuda_ep_moe_block_dev(layer, T, v(d_h), v(d_out), v(d_idx),
                                                      v(d_w), v(stream)))


def moe_block_rep_dev(layer: int, T: int, d_h: int, d_out: int, d_idx: int = 0, d_w: int = 0,
                      stream: int = 0):
    """T tokens every rank holds through the expert-parallel MoE block."""
    v = lambda p: C.c_void_p(int(p) or None)
    _check(load_library().waste_cuda_ep_moe_block_rep_dev(layer, T, v(d_h), v(d_out),
                                                          v(d_idx), v(d_w), v(stream)))
