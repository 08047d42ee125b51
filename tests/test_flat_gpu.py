"""GPU parity of the flat exact search (K1 tensor-core u8 scan and K1g fp32 scan) against the oracle.

The bar is bit-exact: identical ids in identical order and identical f32
distances, for every query.
"""
import ctypes as C
import json
from pathlib import Path

import numpy as np
import pytest

from oracle import pxo
from proxima_b200 import _native as N
from proxima_b200 import fixtures
from proxima_b200.core import Metric, VectorSpace
from proxima_b200.errors import Configuration, DimensionMismatch, DuplicateId, UnknownId

pytestmark = pytest.mark.gpu
KAT = json.loads((Path(__file__).parent / "golden" / "reference_kat.json").read_text())


def _index(dim, metric, **kw):
    from proxima_b200.index import FlatIndex
    return FlatIndex(VectorSpace(dim, metric), **kw)


def _assert_same(gpu, ref, nq):
    gi, gd, gl = gpu
    ri, rd, rl = ref
    assert np.array_equal(gl[:nq], rl[:nq]), "lengths differ"
    for q in range(nq):
        n = int(rl[q])
        assert np.array_equal(gi[q, :n], ri[q, :n]), f"query {q}: ids {gi[q, :n]} vs {ri[q, :n]}"
        assert np.array_equal(gd[q, :n].view(np.uint32), rd[q, :n].view(np.uint32)), f"query {q}: distances"


# ---------------- reference golden cases through the VectorIndex mirror ----------------

def test_golden_flat_cases():
    t = KAT["flat_ties"]
    idx = _index(2, Metric.EUCLIDEAN)
    for i in t["insert_ids"]:
        idx.insert(i, t["vector"])
    assert [h.id for h in idx.search_all(t["vector"], t["k"])] == t["expected_ids"]

    f = KAT["flat_filter"]
    idx = _index(1, Metric.EUCLIDEAN)
    for i in range(f["n"]):
        idx.insert(i, [float(i)], {"keep": i % f["keep_every"] == 0})
    hits = idx.search([0.0], f["k"], lambda _id, m: m.get("keep") is True)
    assert [h.id for h in hits] == f["expected_ids"]

    c = KAT["flat_cosine"]
    idx = _index(2, Metric.COSINE)
    idx.insert(1, c["insert"])
    v = idx.vector(1)
    assert abs(v[0] - c["stored"][0]) < c["tolerance"] and abs(v[1] - c["stored"][1]) < c["tolerance"]
    a = idx.search_all([30.0, 40.0], 1)[0].distance
    b = idx.search_all([0.3, 0.4], 1)[0].distance
    assert abs(a - b) < 1e-6

    g = KAT["flat_k_larger_than_index"]
    idx = _index(1, Metric.EUCLIDEAN)
    for i in range(g["n"]):
        idx.insert(i, [float(i)])
    assert len(idx.search_all([0.0], g["k"])) == g["expected_len"]
    assert idx.search_all([0.0], 0) == []

    tf = KAT["flat_try_from"]
    from proxima_b200.index import FlatIndex
    idx = FlatIndex.from_array(VectorSpace(2, Metric.EUCLIDEAN), tf["data"])
    assert idx.search_all(tf["query"], 1)[0].id == tf["expected_id"]


def test_vector_index_contract():
    idx = _index(3, Metric.EUCLIDEAN)
    assert idx.search_all([1.0, 2.0, 3.0], 10) == []  # empty index: nothing, no error
    idx.insert(1, [3.0, 4.0, 0.0])
    with pytest.raises(DuplicateId):
        idx.insert(1, [1.0, 1.0, 1.0])
    with pytest.raises(DimensionMismatch):
        idx.insert(2, [1.0])
    with pytest.raises(DimensionMismatch):
        idx.search_all([1.0, 2.0], 1)
    with pytest.raises(Configuration):
        idx.search_all([1.0, 2.0, 3.0], (1 << 24) + 1)
    assert idx.search_all([3.0, 4.0, 0.0], 1)[0].distance == 0.0
    idx.upsert(1, [1.0, 1.0, 1.0])
    assert list(idx.vector(1)) == [1.0, 1.0, 1.0] and idx.len() == 1
    idx.remove(1)
    with pytest.raises(UnknownId):
        idx.remove(1)
    assert idx.is_empty() and idx.search_all([1.0, 1.0, 1.0], 3) == []
    # slot churn: removal recycles slots LIFO and results follow the live set
    for i in range(8):
        idx.insert(i, [float(i)] * 3)
    for r in range(50):
        idx.remove(r % 8)
        idx.insert(r % 8, [float(r)] * 3)
    ids = {h.id for h in idx.search_all([0.0, 0.0, 0.0], 8)}
    assert ids == set(range(8))
    assert idx.stats().len == 8 and idx.stats().deleted == 0


# ---------------- C1: quickstart, cosine, 5000 x 64 ----------------

def test_c1_quickstart_bit_exact():
    data = fixtures.quickstart()
    space = VectorSpace(64, Metric.COSINE)
    from proxima_b200.index import FlatIndex
    idx = FlatIndex.from_array(space, data)
    queries = space.prepare_batch(data[::50])
    got = idx.search_prepared_batch(queries, 10)
    ref = pxo.flat_search(pxo.prepare(pxo.COSINE, data), queries, 10, pxo.COSINE)
    assert idx.device_path() == 2  # the f16 screen; unproven queries run on the fp32 scan
    _assert_same(got, ref, 100)
    golden = json.loads((Path(__file__).parent / "golden" / "c1_top10.json").read_text())
    assert [list(map(int, r)) for r in got[0]] == golden["ids"]
    assert [[float(x) for x in r] for r in got[1]] == golden["distances"]


# ---------------- C2 shape: integer blobs, euclidean ----------------

@pytest.fixture(scope="module")
def c2_small():
    db = fixtures.blobs_u8(60_000, 128, 1024, fixtures.C2_CENTRES, fixtures.C2_BASE)
    q = fixtures.blobs_u8(300, 128, 1024, fixtures.C2_CENTRES, fixtures.C2_QUERIES)
    return db, q


@pytest.mark.parametrize("k", [1, 10, 16, 32])
def test_c2_tensor_core_path_bit_exact(c2_small, k):
    db, q = c2_small
    from proxima_b200.index import FlatIndex
    idx = FlatIndex.from_array(VectorSpace(128, Metric.EUCLIDEAN), db)
    assert idx.device_path() == 1
    got = idx.search_prepared_batch(q, k)
    ref = pxo.flat_search(db, q, k, pxo.EUCLIDEAN)
    _assert_same(got, ref, len(q))


def test_c2_many_waves_seeding_and_cross_split_ties():
    """More CTAs than SMs, so later splits seed from finished ones; duplicated rows
    placed in many different splits make exact distance ties cross split borders."""
    db = fixtures.blobs_u8(200_000, 128, 1024, fixtures.C2_CENTRES, fixtures.C2_BASE)
    q = fixtures.blobs_u8(2600, 128, 1024, fixtures.C2_CENTRES, fixtures.C2_QUERIES)
    rows = db.copy()
    src = q[:40]  # the first 40 queries each get 6 exact copies of themselves spread over the store
    for i in range(40):
        for c in range(6):
            rows[(i * 4999 + c * 33_331) % len(rows)] = src[i]
    from proxima_b200.index import FlatIndex
    idx = FlatIndex.from_array(VectorSpace(128, Metric.EUCLIDEAN), rows)
    assert idx.device_path() == 1
    for k in (4, 10):
        got = idx.search_prepared_batch(q, k)
        ref = pxo.flat_search(rows, q, k, pxo.EUCLIDEAN)
        _assert_same(got, ref, len(q))


@pytest.mark.parametrize("k", [33, 64, 100, 128])
def test_c2_grouped_tensor_core_path_bit_exact(c2_small, k):
    """32 < k <= 128: K1 over disjoint row groups, merged, proven exact per query."""
    db, q = c2_small
    from proxima_b200.index import FlatIndex
    idx = FlatIndex.from_array(VectorSpace(128, Metric.EUCLIDEAN), db)
    assert idx.device_path() == 1
    got = idx.search_prepared_batch(q, k)
    ref = pxo.flat_search(db, q, k, pxo.EUCLIDEAN)
    _assert_same(got, ref, len(q))
    assert idx.last_redone() <= 3  # no collect row overflows; blob rows are spread over the groups


def test_c2_grouped_large_batch_runs_in_chunks(c2_small):
    """More than 8,192 queries at 32 < k <= 128 run in chunks of 8,192 (each with
    its own sample pass and collect launch); results stay exact across the
    chunk boundary."""
    db, _ = c2_small
    q = fixtures.blobs_u8(8192 + 300, 128, 1024, fixtures.C2_CENTRES, fixtures.C2_QUERIES)
    from proxima_b200.index import FlatIndex
    idx = FlatIndex.from_array(VectorSpace(128, Metric.EUCLIDEAN), db)
    gi, gd, gl = idx.search_prepared_batch(q, 48)
    pick = np.unique(np.concatenate([np.arange(0, len(q), 97), np.arange(8150, 8250), np.arange(len(q) - 40, len(q))]))
    ri, rd, rl = pxo.flat_search(db, q[pick], 48, pxo.EUCLIDEAN)
    _assert_same((gi[pick], gd[pick], gl[pick]), (ri, rd, rl), len(pick))


def test_c2_grouped_redo_when_neighbours_share_a_group(c2_small):
    """Queries whose top 100 crowd into one row group (40 exact copies in consecutive
    ids) fail the group launches' proof and are answered by the fp32 scan; the
    collect launch (the default) needs no proof and answers all but those whose
    candidate segments overflow. All stay exact."""
    db, q = c2_small
    rows = db[:40_000].copy()
    for i in range(24):
        rows[1000 + i * 1200:1000 + i * 1200 + 40] = q[i]
    from proxima_b200.index import Context, FlatIndex
    ref = pxo.flat_search(rows, q[:200], 100, pxo.EUCLIDEAN)
    ctx = Context(0)
    ctx.set_option("flat_collect_cap", 0)  # the group launches
    idx = FlatIndex.from_array(VectorSpace(128, Metric.EUCLIDEAN), rows, ctx=ctx)
    _assert_same(idx.search_prepared_batch(q[:200], 100), ref, 200)
    assert idx.last_redone() >= 24
    idx = FlatIndex.from_array(VectorSpace(128, Metric.EUCLIDEAN), rows)
    _assert_same(idx.search_prepared_batch(q[:200], 100), ref, 200)
    assert idx.last_redone() < 24  # only queries whose candidate segments overflowed
    # small stores (fewer tiles than groups) take the fp32 scan directly
    small = FlatIndex.from_array(VectorSpace(128, Metric.EUCLIDEAN), db[:700])
    got = small.search_prepared_batch(q[:50], 128)
    ref = pxo.flat_search(db[:700], q[:50], 128, pxo.EUCLIDEAN)
    _assert_same(got, ref, 50)


@pytest.mark.parametrize("sample,cap", [(-1, 2048), (0, 2048), (1, 2048), (4, 2048), (64, 2048), (4, 0), (4, 32),
                                        (-1, 256)])
def test_c2_grouped_shared_bound_sample_pass(c2_small, sample, cap):
    """32 < k <= 128. The sample pass (1/sample of the rows, -1 = 800/k, 0 =
    none) gives the bound T that the single collect launch (cap slots per
    query) or the group launches (cap 0) start from; with cap 32 every query
    overflows its slots and is answered again by the group launches. Results
    stay exact at any setting, also when many rows tie T exactly (copies of a
    query spread over every group) and when the rows are stored sorted (a
    sample far from a query's neighbours, many overflows)."""
    db, q = c2_small
    from proxima_b200.index import Context, FlatIndex
    ctx = Context(0)  # a context of its own: the options stay off the shared default one
    ctx.set_option("flat_group_sample", sample)
    ctx.set_option("flat_collect_cap", cap)
    idx = FlatIndex.from_array(VectorSpace(128, Metric.EUCLIDEAN), db, ctx=ctx)
    for k in (33, 100, 128):
        got = idx.search_prepared_batch(q[:128], k)
        ref = pxo.flat_search(db, q[:128], k, pxo.EUCLIDEAN)
        _assert_same(got, ref, 128)
    rows = db.copy()
    rows[::97] = q[0]  # 619 copies of query 0: its top 128 all tie at distance 0
    rows[50::89] = q[1] + (q[1] < 255)  # near copies of query 1 at one equal distance
    tie = FlatIndex.from_array(VectorSpace(128, Metric.EUCLIDEAN), rows, ctx=ctx)
    for k in (100, 128):
        got = tie.search_prepared_batch(q[:64], k)
        ref = pxo.flat_search(rows, q[:64], k, pxo.EUCLIDEAN)
        _assert_same(got, ref, 64)
    if cap == 32 and sample:
        assert tie.last_redone() >= 64  # every query's candidates overflowed
    order = np.lexsort(db.T[::-1])  # rows sorted: neighbours sit together in id order
    srt = FlatIndex.from_array(VectorSpace(128, Metric.EUCLIDEAN), db[order], ctx=ctx)
    got = srt.search_prepared_batch(q[:96], 100)
    ref = pxo.flat_search(db[order], q[:96], 100, pxo.EUCLIDEAN)
    _assert_same(got, ref, 96)


def test_c2_shuffled_ids_removed_slots_and_duplicates(c2_small):
    db, q = c2_small
    rng = np.random.default_rng(11)
    n = 20_000
    rows = db[:n].copy()
    rows[5000:5400] = rows[100]  # 400 exact duplicates: distance ties resolved by id
    ids = rng.permutation(np.arange(10_000_000, 10_000_000 + n)).astype(np.uint64)
    live = np.ones(n, np.uint8)
    live[rng.choice(n, 1500, replace=False)] = 0
    from proxima_b200.index import Context
    ctx = Context.default()
    h = N.vp()
    N.call("pxc_flat_create", ctx.handle, 128, 0, C.byref(h))
    try:
        N.call("pxc_flat_sync", h, N.ptr(rows), N.ptr(ids), N.ptr(live), 0, n)
        assert N.load().pxc_flat_path(h) == 1
        queries = np.concatenate([q[:200], rows[100:101]])
        for k in (10, 32):
            out = (np.zeros((len(queries), k), np.uint64), np.zeros((len(queries), k), np.float32),
                   np.zeros(len(queries), np.uint32))
            N.call("pxc_flat_search", h, N.ptr(queries), len(queries), k, None, *map(N.ptr, out))
            ref = pxo.flat_search(rows, queries, k, pxo.EUCLIDEAN, ids=ids, live=live)
            _assert_same(out, ref, len(queries))
    finally:
        N.load().pxc_flat_destroy(h)


def test_c2_filtered_and_non_integer(c2_small):
    db, q = c2_small
    n = 30_000
    rows = db[:n]
    keep = (np.arange(n) % 7) == 3
    bitmap = np.packbits(keep, bitorder="little")
    bitmap = np.concatenate([bitmap, np.zeros(-len(bitmap) % 8, np.uint8)]).view(np.uint64)
    from proxima_b200.index import FlatIndex
    idx = FlatIndex.from_array(VectorSpace(128, Metric.EUCLIDEAN), rows)
    got = idx.search_prepared_batch(q[:64], 10, bitmap)
    ref = pxo.flat_search(rows, q[:64], 10, pxo.EUCLIDEAN, bitmap=bitmap)
    _assert_same(got, ref, 64)
    # non-integer queries on an integer store fall back to the fp32 scan, still exact
    qf = q[:64] + np.float32(0.25)
    got = idx.search_prepared_batch(qf, 10)
    ref = pxo.flat_search(rows, qf, 10, pxo.EUCLIDEAN)
    _assert_same(got, ref, 64)


def _bitmap(keep):
    bm = np.packbits(keep, bitorder="little")
    return np.concatenate([bm, np.zeros(-len(bm) % 8, np.uint8)]).view(np.uint64)


@pytest.mark.parametrize("k", [1, 10, 32, 100])
def test_c2_filtered_tensor_core_path_bit_exact(c2_small, k):
    """A filter on an integer euclidean store runs on the tensor-core scan over
    the accepted rows; ids not in slot order and dead slots included."""
    db, q = c2_small
    n = 60_000
    rows = db[:n]
    rng = np.random.default_rng(k)
    ids = rng.permutation(n).astype(np.uint64) * 5 + 3
    live = (rng.random(n) > 0.1).astype(np.uint8)
    h = N.vp()
    from proxima_b200.index import Context
    ctx = Context.default()
    N.call("pxc_flat_create", ctx.handle, 128, 0, C.byref(h))
    N.call("pxc_flat_sync", h, N.ptr(rows), N.ptr(ids), N.ptr(live), 0, n)
    nq = 300
    for keep in ((rng.random(n) < 0.1), (np.arange(n) % 2 == 0), np.zeros(n, bool), np.ones(n, bool),
                 (np.arange(n) < 5)):
        bm = _bitmap(keep)
        oid = np.zeros((nq, k), np.uint64)
        od = np.zeros((nq, k), np.float32)
        ol = np.zeros(nq, np.uint32)
        N.call("pxc_flat_search", h, N.ptr(q[:nq]), nq, k, N.ptr(bm), N.ptr(oid), N.ptr(od), N.ptr(ol))
        assert N.load().pxc_flat_path(h) == 1
        ref = pxo.flat_search(rows, q[:nq], k, pxo.EUCLIDEAN, ids=ids, live=live, bitmap=bm)
        _assert_same((oid, od, ol), ref, nq)
    N.load().pxc_flat_destroy(h)


@pytest.mark.parametrize("metric", [Metric.EUCLIDEAN, Metric.INNER_PRODUCT, Metric.MANHATTAN, Metric.COSINE])
@pytest.mark.parametrize("dim", [3, 37, 96])
def test_generic_metrics_bit_exact(metric, dim):
    rng = np.random.default_rng(dim * 10 + int(metric))
    rows = (rng.standard_normal((7000, dim)) * 2).astype(np.float32)
    qs = (rng.standard_normal((45, dim)) * 2).astype(np.float32)
    space = VectorSpace(dim, metric)
    from proxima_b200.index import FlatIndex
    idx = FlatIndex.from_array(space, rows)
    pq = space.prepare_batch(qs)
    for k in (1, 17, 300):
        got = idx.search_prepared_batch(pq, k)
        ref = pxo.flat_search(pxo.prepare(int(metric), rows), pq, k, int(metric))
        _assert_same(got, ref, len(qs))


def test_large_k_uses_segmented_sort():
    rng = np.random.default_rng(2)
    rows = rng.standard_normal((5000, 8)).astype(np.float32)
    qs = rng.standard_normal((3, 8)).astype(np.float32)
    from proxima_b200.index import FlatIndex
    idx = FlatIndex.from_array(VectorSpace(8, Metric.EUCLIDEAN), rows)
    got = idx.search_prepared_batch(qs, 4500)
    ref = pxo.flat_search(rows, qs, 4500, pxo.EUCLIDEAN)
    _assert_same(got, ref, 3)


def test_topk_merge_of_shards_equals_single_search(c2_small):
    """Row shards searched separately (as ranks do) and merged == one search."""
    db, q = c2_small
    import torch
    from proxima_b200.index import Context
    ctx = Context.default()
    n, k, parts = 40_000, 10, 4
    qs = q[:130]
    ids_all, d_all, l_all = [], [], []
    for p in range(parts):
        lo, hi = p * n // parts, (p + 1) * n // parts
        h = N.vp()
        N.call("pxc_flat_create", ctx.handle, 128, 0, C.byref(h))
        gids = np.arange(lo, hi, dtype=np.uint64)
        N.call("pxc_flat_sync", h, N.ptr(db[lo:hi]), N.ptr(gids), None, 0, hi - lo)
        out = (np.zeros((len(qs), k), np.uint64), np.zeros((len(qs), k), np.float32), np.zeros(len(qs), np.uint32))
        N.call("pxc_flat_search", h, N.ptr(qs), len(qs), k, None, *map(N.ptr, out))
        N.load().pxc_flat_destroy(h)
        ids_all.append(out[0]); d_all.append(out[1]); l_all.append(out[2])
    dev = torch.device("cuda:0")
    t_ids = torch.from_numpy(np.stack(ids_all).view(np.int64)).to(dev)
    t_d = torch.from_numpy(np.stack(d_all)).to(dev)
    t_l = torch.from_numpy(np.stack(l_all).view(np.int32)).to(dev)
    o_ids = torch.zeros((len(qs), k), dtype=torch.int64, device=dev)
    o_d = torch.zeros((len(qs), k), dtype=torch.float32, device=dev)
    o_l = torch.zeros(len(qs), dtype=torch.int32, device=dev)
    N.call("pxc_topk_merge", ctx.handle, t_ids.data_ptr(), t_d.data_ptr(), t_l.data_ptr(), parts, len(qs), k, k,
           o_ids.data_ptr(), o_d.data_ptr(), o_l.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    got = (o_ids.cpu().numpy().view(np.uint64), o_d.cpu().numpy(), o_l.cpu().numpy().view(np.uint32))
    ref = pxo.flat_search(db[:n], qs, k, pxo.EUCLIDEAN)
    _assert_same(got, ref, len(qs))


def test_c2_many_query_tiles_match_brute_force():
    """Thousands of queries: the scan runs in several waves, later splits seed
    their lists from finished ones (including lists that were seeded
    themselves). Checked against a brute-force scan in exact integer
    arithmetic, ties by id."""
    import torch

    from proxima_b200 import _native as N
    from proxima_b200 import fixtures

    n, dim, nq, k = 300_000, 128, 4096, 10
    db = fixtures.blobs_u8(n, dim, 512, fixtures.C2_CENTRES, fixtures.C2_BASE)
    q = fixtures.blobs_u8(nq, dim, 512, fixtures.C2_CENTRES, fixtures.C2_QUERIES)
    from proxima_b200.index import Context
    import ctypes as C

    ctx = Context.default()
    h = N.vp()
    N.call("pxc_flat_create", ctx.handle, dim, 0, C.byref(h))
    try:
        N.call("pxc_flat_sync", h, N.ptr(db), None, None, 0, n)
        assert N.load().pxc_flat_path(h) == 1
        ids = np.zeros((nq, k), np.uint64)
        dist = np.zeros((nq, k), np.float32)
        lens = np.zeros(nq, np.uint32)
        N.call("pxc_flat_search", h, N.ptr(q), nq, k, None, N.ptr(ids), N.ptr(dist), N.ptr(lens))
        dbt = torch.from_numpy(db).cuda().to(torch.int64)
        qt = torch.from_numpy(q).cuda().to(torch.int64)
        for i in list(range(0, nq, 97)) + [nq - 1]:
            d = ((dbt - qt[i]) ** 2).sum(1)
            kth = torch.topk(d, k, largest=False).values.max()
            cand = torch.nonzero(d <= kth).flatten()
            order = sorted(zip(d[cand].tolist(), cand.tolist()))[:k]
            assert lens[i] == k
            assert ids[i].tolist() == [c for _, c in order], f"query {i}: ids"
            assert dist[i].tolist() == [float(v) for v, _ in order], f"query {i}: distances"
    finally:
        N.load().pxc_flat_destroy(h)


def test_c1_reproduces_the_reference_transcript():
    """The reference's README prints the quickstart's run (README.md, "60-second
    quickstart"): the filtered search of the first query (lang == "en", k = 10)
    answers "10 hits, nearest 0 at 0.0000". The exact flat index over the same
    5,000 vectors and metadata (every third id "en") must print the same line;
    this pins C1 to output of the reference itself, not to the oracle."""
    from proxima_b200.filters import MetadataFilter
    from proxima_b200.index import FlatIndex
    data = fixtures.quickstart()
    idx = FlatIndex(VectorSpace(64, Metric.COSINE), capacity=5000)
    for i in range(5000):
        idx.insert(i, data[i], {"lang": "en" if i % 3 == 0 else "fr"})
    hits = idx.search(data[0], 10, MetadataFilter.parse({"lang": "en"}))
    line = f"{len(hits)} hits, nearest {hits[0].id} at {hits[0].distance:.4f}"
    assert line == "10 hits, nearest 0 at 0.0000"
    assert all(h.id % 3 == 0 for h in hits)
    idx.close()
