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
    _same(_sharded_search("pxc_flat_search_sharded_owned", h, ctx, q, 10), ref, "owned, one rank")
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
            # the owner-computes exchange: this rank's slice of the same batch
            b, oi, od, ol = sh.search_owned(torch.from_numpy(qh).cuda(), 10, torch.cuda.current_stream().cuda_stream)
            torch.cuda.synchronize()
            sh.close()
            ri, rd, rl = pxo.flat_search(data, qh, 10, int(metric))
            n = oi.shape[0]
            own_ok = bool(n == (len(qh) * (rank + 1)) // world - b and b == (len(qh) * rank) // world and
                          np.array_equal(ol.cpu().numpy().view(np.uint32), rl[b:b + n]) and
                          np.array_equal(oi.cpu().numpy().view(np.uint64), ri[b:b + n]) and
                          np.array_equal(od.cpu().numpy().view(np.uint32), rd[b:b + n].view(np.uint32)))
            flag = torch.tensor([1 if own_ok else 0], dtype=torch.int32, device="cuda")
            dist.all_reduce(flag, op=dist.ReduceOp.MIN)
            results[label + " owned"] = bool(flag.item() == 1)
            if rank == 0:
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
    assert res == {"u8": True, "real cosine": True, "u8 owned": True, "real cosine owned": True}, res


def _merge_by_total_order(parts, k):
    """Union of per-shard (ids, dist, len) answers ordered by (total_cmp(distance), id), first k."""
    nq = parts[0][0].shape[0]
    ids = np.zeros((nq, k), np.uint64)
    dist = np.zeros((nq, k), np.float32)
    lens = np.zeros(nq, np.uint32)
    for q in range(nq):
        cand = []
        for pi, pd, pl in parts:
            for j in range(int(pl[q])):
                b = int(pd[q, j:j + 1].view(np.int32)[0])
                key = b ^ 0x7FFFFFFF if b < 0 else b
                cand.append((key, int(pi[q, j]), pd[q, j]))
        cand.sort(key=lambda c: (c[0], c[1]))
        cand = cand[:k]
        lens[q] = len(cand)
        for j, c in enumerate(cand):
            ids[q, j], dist[q, j] = c[1], c[2]
    return ids, dist, lens


def _ivf_shard_answer(data, lo, hi, cent, books, m, queries, k, nprobe, rerank):
    from oracle import pxo

    rows = data[lo:hi]
    list_of = np.zeros(len(rows), np.uint32)
    codes = np.zeros((len(rows), m), np.uint8)
    pxo.lib().pxo_ivfpq_encode_all(rows.ctypes.data, None, len(rows), rows.shape[1], cent.ctypes.data, len(cent),
                                   books.ctypes.data, m, list_of.ctypes.data, codes.ctypes.data, pxo.threads())
    return pxo.ivfpq_search(rows, cent, books, m, list_of, codes, queries, k, nprobe, rerank,
                            ids=np.arange(lo, hi, dtype=np.uint64))


def test_single_rank_ivfpq_sharded_equals_search():
    from oracle import pxo
    from proxima_b200 import _native as N
    from proxima_b200 import fixtures
    from proxima_b200.index import Context
    from proxima_b200.ivfpq import IvfPqIndex

    ctx = Context(0)
    N.call("pxc_ctx_init_comm", ctx.handle, (C.c_uint8 * 128)(), 1, 0, 5000)
    data = fixtures.blobs_u8(20_000, 32, 64, 3, 4) + np.float32(0.25)
    queries = fixtures.blobs_u8(200, 32, 64, 3, 5)
    cent, books, _, _, _ = pxo.ivfpq_train(data, 64, 8, 4, 10_000, 0x77)
    idx = IvfPqIndex(32, 64, 8, context=ctx)
    idx.from_parts(cent, books)
    idx.set_store(data, ids=np.arange(500, 500 + len(data), dtype=np.uint64))
    idx.encode_all()
    q = torch.from_numpy(queries).cuda()
    out = [torch.empty((200, 10), dtype=torch.int64, device="cuda"), torch.empty((200, 10), device="cuda"),
           torch.empty(200, dtype=torch.int32, device="cuda")]
    idx.search_sharded_device(q, 10, 6, 50, *out, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    ref = _ivf_shard_answer(data, 0, len(data), cent, books, 8, queries, 10, 6, 50)
    ref = (ref[0] + np.uint64(500), ref[1], ref[2])
    _same((out[0].cpu().numpy().view(np.uint64), out[1].cpu().numpy(), out[2].cpu().numpy().view(np.uint32)), ref,
          "ivf-pq sharded, one rank")
    idx.close()
    ctx.close()


def _ivf_rank(rank, world, port, out):
    import sys

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    from datetime import timedelta

    from oracle import pxo
    from proxima_b200 import fixtures
    from proxima_b200.index import Context
    from proxima_b200.ivfpq import IvfPqIndex
    from proxima_b200.sharded import init_comm, shard_range

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        ctx = Context(rank)
        init_comm(ctx, timeout_ms=30_000)
        data = fixtures.blobs_u8(40_000, 32, 64, 3, 4)
        queries = fixtures.blobs_u8(300, 32, 64, 3, 5)
        cent, books, _, _, _ = pxo.ivfpq_train(data, 64, 8, 4, 10_000, 0x77)  # replicated parts
        lo, hi = shard_range(len(data), rank, world)
        idx = IvfPqIndex(32, 64, 8, context=ctx)
        idx.from_parts(cent, books)
        idx.set_store(data[lo:hi], ids=np.arange(lo, hi, dtype=np.uint64))
        idx.encode_all()
        q = torch.from_numpy(queries).cuda()
        res = [torch.empty((300, 10), dtype=torch.int64, device="cuda"), torch.empty((300, 10), device="cuda"),
               torch.empty(300, dtype=torch.int32, device="cuda")]
        idx.search_sharded_device(q, 10, 8, 100, *res, torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        if rank == 0:
            parts = [_ivf_shard_answer(data, *shard_range(len(data), r, world), cent, books, 8, queries, 10, 8, 100)
                     for r in range(world)]
            ri, rd, rl = _merge_by_total_order(parts, 10)
            gi = res[0].cpu().numpy().view(np.uint64)
            gd = res[1].cpu().numpy()
            gl = res[2].cpu().numpy().view(np.uint32)
            out.put(bool(np.array_equal(gl, rl) and np.array_equal(gi, ri) and
                         np.array_equal(gd.view(np.uint32), rd.view(np.uint32))))
        idx.close()
        ctx.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_two_rank_sharded_ivfpq_equals_the_oracle_composition():
    """Lists split by rows over two ranks, each probing the same lists on its
    shard with its own shortlist, then the exchange: equal to the oracle's
    per-shard search_prepared merged by (total_cmp, id)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    mctx = mp.get_context("spawn")
    q = mctx.Queue()
    port = _free_port()
    procs = [mctx.Process(target=_ivf_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(240)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert q.get(timeout=10) is True


def test_single_rank_sharded_kmeans_equals_kmeans():
    """One rank: the sharded k-means (exchanges included) is the unsharded run
    bit for bit, empty-cluster re-seeding included (duplicated init rows)."""
    from proxima_b200 import _native as N
    from proxima_b200 import fixtures
    from proxima_b200.index import Context
    from proxima_b200.quantize import kmeans, kmeans_sharded

    ctx = Context(0)
    N.call("pxc_ctx_init_comm", ctx.handle, (C.c_uint8 * 128)(), 1, 0, 5000)
    pts = fixtures.sphere_blobs(20_000, 48, 60, 21, 22, 0.05)
    init = pts[:300].copy()
    init[150:200] = init[100:150]  # duplicates: the higher copies end empty and are re-seeded
    d = torch.from_numpy(pts).cuda()
    a = kmeans(d, 48, 300, 8, init=init, context=ctx, want_assignment=True)
    b = kmeans_sharded(d, 48, 300, 8, init, ctx)
    assert b.reseeded > 0 and a.reseeded == b.reseeded
    assert a.iterations == b.iterations and a.inertia == b.inertia
    assert np.array_equal(a.centroids.view(np.uint32), b.centroids.view(np.uint32))
    assert np.array_equal(a.assignment, b.assignment)
    ctx.close()


def _km_rank(rank, world, port, out):
    import sys

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    from datetime import timedelta

    from oracle import pxo
    from proxima_b200 import fixtures
    from proxima_b200.index import Context
    from proxima_b200.quantize import kmeans_sharded
    from proxima_b200.sharded import init_comm, shard_range

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        ctx = Context(rank)
        init_comm(ctx, timeout_ms=30_000)
        pts = fixtures.sphere_blobs(60_000, 64, 200, 31, 32, 0.05)
        init = pts[:512].copy()
        init[300:340] = init[200:240]  # empty clusters to re-seed across the ranks
        lo, hi = shard_range(len(pts), rank, world)
        got = kmeans_sharded(torch.from_numpy(pts[lo:hi]).cuda(), 64, 512, 10, init, ctx)
        assigns = [torch.empty(shard_range(len(pts), r, world)[1] - shard_range(len(pts), r, world)[0],
                               dtype=torch.int32, device="cuda") for r in range(world)]
        dist.all_gather(assigns, torch.from_numpy(got.assignment.view(np.int32)).cuda())
        if rank == 0:
            cent, assign, inertia, iters = pxo.kmeans(pts, 512, 10, init=init)
            ga = np.concatenate([a.cpu().numpy().view(np.uint32) for a in assigns])
            rel = np.abs(got.centroids - cent).max() / max(np.abs(cent).max(), 1e-30)
            out.put({"iterations": got.iterations == iters, "reseeded": got.reseeded > 0,
                     "assign_diff": int((ga != assign).sum()), "centroid_rel": float(rel),
                     "inertia_rel": abs(got.inertia - inertia) / inertia})
        ctx.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_two_rank_sharded_kmeans_matches_the_oracle():
    """Points split over two ranks: the same iterations, re-seeds and
    assignments as the oracle's kmeans over all points, centroids within 1e-3
    relative (the per-cluster f64 sums are folded in rank order)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    mctx = mp.get_context("spawn")
    q = mctx.Queue()
    port = _free_port()
    procs = [mctx.Process(target=_km_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(240)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = q.get(timeout=10)
    assert res["iterations"] and res["reseeded"], res
    assert res["assign_diff"] <= 60 and res["centroid_rel"] < 1e-3 and res["inertia_rel"] < 1e-6, res
