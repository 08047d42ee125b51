"""The library's multi-GPU search: the context's NCCL communicator, the row-
sharded flat search and the generic candidate exchange, against the oracle's
unsharded FlatIndex::search (crates/proxima-index/src/flat.rs:153-169), bit
for bit. One rank runs on any GPU box; two ranks run as child processes when
the box has two GPUs (NVLS off, per-process GPU), otherwise that case skips.
"""
import ctypes as C
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _same(got, ref, label):
    gi, gd, gl = got
    ri, rd, rl = ref
    assert np.array_equal(gl, rl), f"{label}: lengths"
    for q in range(len(rl)):
        n = int(rl[q])
        assert np.array_equal(gi[q, :n], ri[q, :n]), f"{label} query {q}: ids"
        assert np.array_equal(gd[q, :n].view(np.uint32), rd[q, :n].view(np.uint32)), f"{label} query {q}: distances"


def _sharded_search(entry, handle, ctx, q, k):
    from proxima_b200 import _native as N

    nq = q.shape[0]
    ids = torch.empty((nq, k), dtype=torch.int64, device="cuda")
    d = torch.empty((nq, k), dtype=torch.float32, device="cuda")
    ln = torch.empty(nq, dtype=torch.int32, device="cuda")
    N.call(entry, handle, q.data_ptr(), nq, k, None, ids.data_ptr(), d.data_ptr(), ln.data_ptr(),
           torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return ids.cpu().numpy().view(np.uint64), d.cpu().numpy(), ln.cpu().numpy().view(np.uint32)


def test_single_rank_communicator_and_exchange():
    """nranks = 1: the sharded search and the exchange reduce to a local merge."""
    from oracle import pxo
    from proxima_b200 import _native as N
    from proxima_b200 import fixtures
    from proxima_b200.index import Context

    ctx = Context(0)
    N.call("pxc_ctx_init_comm", ctx.handle, (C.c_uint8 * 128)(), 1, 0, 5000)
    assert N.load().pxc_ctx_comm_size(ctx.handle) == 1 and N.load().pxc_ctx_comm_rank(ctx.handle) == 0
    db = fixtures.blobs_u8(30_000, 64, 128, 5, 6)
    qh = fixtures.blobs_u8(300, 64, 128, 5, 7)
    h = N.vp()
    N.call("pxc_flat_create", ctx.handle, 64, 0, C.byref(h))
    ids = np.arange(1000, 1000 + len(db), dtype=np.uint64)
    N.call("pxc_flat_sync", h, N.ptr(db), N.ptr(ids), None, 0, len(db))
    q = torch.from_numpy(qh).cuda()
    got = _sharded_search("pxc_flat_search_sharded", h, ctx, q, 10)
    ref = pxo.flat_search(db, qh, 10, pxo.EUCLIDEAN, ids=ids)
    _same(got, ref, "sharded, one rank")
    # the generic exchange of given lists (k_in = 10 -> k = 7)
    li = torch.from_numpy(got[0].view(np.int64)).cuda()
    ld = torch.from_numpy(got[1]).cuda()
    ll = torch.from_numpy(got[2].view(np.int32)).cuda()
    oi = torch.empty((300, 7), dtype=torch.int64, device="cuda")
    od = torch.empty((300, 7), dtype=torch.float32, device="cuda")
    ol = torch.empty(300, dtype=torch.int32, device="cuda")
    N.call("pxc_topk_exchange", ctx.handle, li.data_ptr(), ld.data_ptr(), ll.data_ptr(), 300, 10, 7, oi.data_ptr(),
           od.data_ptr(), ol.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert np.array_equal(oi.cpu().numpy().view(np.uint64), got[0][:, :7])
    assert np.array_equal(od.cpu().numpy().view(np.uint32), got[1][:, :7].view(np.uint32))
    N.load().pxc_flat_destroy(h)
    ctx.close()


def _rank(rank, world, port, out):
    import sys

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    from datetime import timedelta

    from oracle import pxo
    from proxima_b200 import _native as N
    from proxima_b200 import fixtures
    from proxima_b200.core import Metric, VectorSpace
    from proxima_b200.index import Context
    from proxima_b200.sharded import ShardedFlat, init_comm, shard_range

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        ctx = Context(rank)
        init_comm(ctx, timeout_ms=30_000)
        results = {}
        for label, data, metric in (
                ("u8", fixtures.blobs_u8(50_000, 96, 256, 11, 12), Metric.EUCLIDEAN),
                ("real cosine", fixtures.sphere_blobs(50_000, 96, 256, 11, 13, 0.05), Metric.COSINE)):
            space = VectorSpace(96, metric)
            data = space.prepare_batch(data)
            offset = np.float32(0.001) if metric == Metric.COSINE else np.float32(0.0)  # u8: integer queries (K1)
            qh = space.prepare_batch(data[::97][:400] + offset)
            lo, hi = shard_range(len(data), rank, world)
            sh = ShardedFlat(ctx, 96, int(metric), data[lo:hi], lo)
            got = sh.search_global(torch.from_numpy(qh).cuda(), 10, torch.cuda.current_stream().cuda_stream)
            torch.cuda.synchronize()
            sh.close()
            if rank == 0:
                ri, rd, rl = pxo.flat_search(data, qh, 10, int(metric))
                gi = got[0].cpu().numpy().view(np.uint64)
                gd = got[1].cpu().numpy()
                gl = got[2].cpu().numpy().view(np.uint32)
                results[label] = bool(np.array_equal(gl, rl) and np.array_equal(gi, ri) and
                                      np.array_equal(gd.view(np.uint32), rd.view(np.uint32)))
        if rank == 0:
            out.put(results)
        ctx.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_two_rank_sharded_flat_equals_unsharded():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    mctx = mp.get_context("spawn")
    q = mctx.Queue()
    port = _free_port()
    procs = [mctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(240)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = q.get(timeout=10)
    assert res == {"u8": True, "real cosine": True}, res
