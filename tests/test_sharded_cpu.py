"""Multi-rank path on CPU: row sharding and the candidate allgather over gloo (world size 2).

Each rank computes its shard's top-k with the oracle (the checker), exchanges
candidates through proxima_b200.sharded.exchange_candidates, and rank 0 checks
that merging the gathered lists by (total_cmp, id) equals one unsharded search.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _total_key(d: np.ndarray) -> np.ndarray:
    b = d.astype(np.float32).view(np.int32).astype(np.int64)
    return np.where(b < 0, b ^ 0x7FFFFFFF, b)


def _worker(rank, world, port, n, nq, k, out):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from oracle import pxo
    from proxima_b200 import fixtures
    from proxima_b200.sharded import exchange_candidates, shard_range

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        db = fixtures.blobs_u8(n, 32, 16, 1, 2)
        q = fixtures.blobs_u8(nq, 32, 16, 1, 3)
        lo, hi = shard_range(n, rank, world)
        ids, d, lens = pxo.flat_search(db[lo:hi], q, k, pxo.EUCLIDEAN,
                                       ids=np.arange(lo, hi, dtype=np.uint64), nthreads=1)
        g_ids, g_d, g_l = exchange_candidates(torch.from_numpy(ids.view(np.int64)), torch.from_numpy(d),
                                              torch.from_numpy(lens.view(np.int32)))
        if rank == 0:
            g_ids, g_d, g_l = g_ids.numpy(), g_d.numpy(), g_l.numpy()
            ref_ids, ref_d, _ = pxo.flat_search(db, q, k, pxo.EUCLIDEAN, nthreads=1)
            ok = True
            for qi in range(nq):
                cand = [(int(_total_key(g_d[p, qi, j:j + 1])[0]), int(g_ids[p, qi, j]), float(g_d[p, qi, j]))
                        for p in range(world) for j in range(int(g_l[p, qi]))]
                cand.sort()
                got = [c[1] for c in cand[:k]]
                ok &= got == [int(x) for x in ref_ids[qi]]
            covered = sum(shard_range(n, r, world)[1] - shard_range(n, r, world)[0] for r in range(world))
            out.put((ok, covered == n))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_two_rank_gloo_exchange_merges_to_the_unsharded_answer():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, 3001, 37, 7, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(90)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    ok, covered = q.get(timeout=5)
    assert ok and covered


def test_shard_ranges_partition_rows():
    from proxima_b200.sharded import shard_range

    for n in (0, 1, 7, 1000, 1_000_000):
        for world in (1, 2, 3, 8):
            spans = [shard_range(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert max(h - l for l, h in spans) - min(h - l for l, h in spans) <= 1


def _id_worker(rank, world, port, out):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from proxima_b200.sharded import broadcast_comm_id

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        out.put((rank, broadcast_comm_id()))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_two_rank_gloo_communicator_id_handoff():
    """Rank 0's communicator id (created by the native library, no GPU needed)
    reaches every rank unchanged: what pxc_ctx_init_comm then joins on."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_id_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(90)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    got = dict(q.get(timeout=5) for _ in range(2))
    assert len(got[0]) == 128 and got[0] == got[1] and any(got[0])
