"""Row-sharded exact search across GPUs (one process per GPU).

Each rank mirrors a contiguous range of database rows with their global
VectorIds and joins the job's NCCL communicator, which the native library owns
(``pxc_ctx_init_comm``). ``pxc_flat_search_sharded`` searches every query on the
rank's shard, carries the k (id, distance) candidates per query to every rank in
one packed allgather and merges them on the device. The only data that crosses
NVLink is k candidates per query per rank. ``torch.distributed`` is used only
to hand rank 0's 128-byte communicator id to the other ranks.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch
import torch.distributed as dist

from . import _native as N


def shard_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous rows [lo, hi) of rank `rank` out of `world` (sizes differ by at most 1)."""
    return rank * n // world, (rank + 1) * n // world


def broadcast_comm_id(group=None) -> bytes:
    """Rank 0's fresh communicator id (pxc_comm_unique_id), broadcast to every
    rank of `group` (gloo: CPU tensor; nccl: CUDA tensor)."""
    lib = N.load()
    buf = (C.c_uint8 * 128)()
    if dist.get_rank(group) == 0:
        N.call("pxc_comm_unique_id", buf)
    backend = dist.get_backend(group)
    dev = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")
    t = torch.tensor(list(bytes(buf)), dtype=torch.uint8, device=dev)
    dist.broadcast(t, src=dist.get_global_rank(group, 0) if group is not None else 0, group=group)
    del lib
    return bytes(t.cpu().tolist())


def init_comm(ctx, group=None, timeout_ms: int = 60_000) -> None:
    """Join the context to the communicator of the ranks of `group` (collective)."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    cid = broadcast_comm_id(group)
    idbuf = (C.c_uint8 * 128).from_buffer_copy(cid)
    N.call("pxc_ctx_init_comm", ctx.handle, idbuf, world, rank, timeout_ms)


def exchange_candidates(ids: torch.Tensor, dist_: torch.Tensor, lens: torch.Tensor, group=None):
    """Allgather the per-rank candidate lists through torch.distributed (the host-side
    restatement the CPU tests check the merge semantics with; the GPU path uses
    the library's own exchange).

    ids [nq, k] int64, dist_ [nq, k] float32, lens [nq] int32 -> tensors of shape
    [world, nq, k], [world, nq, k], [world, nq] in rank order (NCCL for CUDA
    tensors, gloo for CPU tensors)."""
    world = dist.get_world_size(group)
    out_ids = [torch.empty_like(ids) for _ in range(world)]
    out_d = [torch.empty_like(dist_) for _ in range(world)]
    out_l = [torch.empty_like(lens) for _ in range(world)]
    dist.all_gather(out_ids, ids.contiguous(), group=group)
    dist.all_gather(out_d, dist_.contiguous(), group=group)
    dist.all_gather(out_l, lens.contiguous(), group=group)
    return torch.stack(out_ids), torch.stack(out_d), torch.stack(out_l)


class ShardedFlat:
    """One rank's shard of a flat index plus the cross-rank merge."""

    def __init__(self, ctx, dim: int, metric: int, rows: np.ndarray, first_id: int):
        self.ctx = ctx
        self.dim = dim
        self.lib = N.load()
        h = N.vp()
        N.call("pxc_flat_create", ctx.handle, dim, metric, C.byref(h))
        self.handle = h
        gids = np.arange(first_id, first_id + rows.shape[0], dtype=np.uint64)
        rows = np.ascontiguousarray(rows, dtype=np.float32)  # a reference held across the call
        N.call("pxc_flat_sync", h, N.ptr(rows), N.ptr(gids),
               None, 0, rows.shape[0])

    def search(self, q_dev: torch.Tensor, k: int, stream_ptr: int):
        nq = q_dev.shape[0]
        dev = q_dev.device
        ids = torch.empty((nq, k), dtype=torch.int64, device=dev)
        d = torch.empty((nq, k), dtype=torch.float32, device=dev)
        lens = torch.empty(nq, dtype=torch.int32, device=dev)
        N.call("pxc_flat_search_device", self.handle, q_dev.data_ptr(), nq, k, None, ids.data_ptr(),
               d.data_ptr(), lens.data_ptr(), stream_ptr)
        return ids, d, lens

    def search_global(self, q_dev: torch.Tensor, k: int, stream_ptr: int):
        """Local search, one packed NCCL allgather, device merge -> global top-k on every rank
        (the context must have joined the communicator: init_comm)."""
        nq = q_dev.shape[0]
        m_ids = torch.empty((nq, k), dtype=torch.int64, device=q_dev.device)
        m_d = torch.empty((nq, k), dtype=torch.float32, device=q_dev.device)
        m_l = torch.empty(nq, dtype=torch.int32, device=q_dev.device)
        N.call("pxc_flat_search_sharded", self.handle, q_dev.data_ptr(), nq, k, None, m_ids.data_ptr(),
               m_d.data_ptr(), m_l.data_ptr(), stream_ptr)
        return m_ids, m_d, m_l

    def search_owned(self, q_dev: torch.Tensor, k: int, stream_ptr: int):
        """Local search of every query, then each rank receives only the candidates of its own
        query slice (pxc_flat_search_sharded_owned): returns (begin, ids, dist, lens) of that slice."""
        nq = q_dev.shape[0]
        b, n = C.c_uint32(), C.c_uint32()
        self.lib.pxc_ctx_owned_range(self.ctx.handle, nq, C.byref(b), C.byref(n))
        m_ids = torch.empty((max(n.value, 1), k), dtype=torch.int64, device=q_dev.device)
        m_d = torch.empty((max(n.value, 1), k), dtype=torch.float32, device=q_dev.device)
        m_l = torch.empty(max(n.value, 1), dtype=torch.int32, device=q_dev.device)
        N.call("pxc_flat_search_sharded_owned", self.handle, q_dev.data_ptr(), nq, k, None, m_ids.data_ptr(),
               m_d.data_ptr(), m_l.data_ptr(), stream_ptr)
        return b.value, m_ids[:n.value], m_d[:n.value], m_l[:n.value]

    def close(self):
        if self.handle:
            self.lib.pxc_flat_destroy(self.handle)
            self.handle = None
