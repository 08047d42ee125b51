"""IVF-PQ search on the GPU (pxc_ivfpq) against the oracle's restatement of
IvfPqIndex::search_prepared (crates/proxima-index/src/ivfpq.rs:998-1110), on
the same trained parts: ids, distances and lengths bit for bit, with and
without reranking, euclidean and cosine, filters, VectorIds that are not the
slot numbers, dead slots, layouts whose widths are not all equal."""
import numpy as np
import pytest

from oracle import pxo
from proxima_b200 import fixtures
from proxima_b200.core import Metric
from proxima_b200.ivfpq import IvfPqIndex

pytestmark = pytest.mark.gpu


def _same(got, ref, label):
    gi, gd, gl = got
    ri, rd, rl = ref
    assert np.array_equal(gl, rl), f"{label}: lengths"
    for q in range(len(rl)):
        n = int(rl[q])
        assert np.array_equal(gi[q, :n], ri[q, :n]), f"{label}: ids of query {q}"
        assert np.array_equal(gd[q, :n].view(np.uint32), rd[q, :n].view(np.uint32)), f"{label}: distances of query {q}"


def _build(n, dim, nlist, m, seed, metric=pxo.EUCLIDEAN, nblobs=64):
    data = fixtures.blobs_u8(n, dim, nblobs, fixtures.C4_CENTRES + seed, fixtures.C4_BASE + seed)
    if metric == pxo.COSINE:
        data = data - 127.5
        data /= np.linalg.norm(data, axis=1, keepdims=True)
        data = data.astype(np.float32)
    cent, books, list_of, codes, _ = pxo.ivfpq_train(data, nlist, m, max_iterations=8, training_sample=5000,
                                                       seed=seed)
    return data, cent, books, list_of, codes


@pytest.mark.parametrize("metric", [pxo.EUCLIDEAN, pxo.COSINE])
def test_search_matches_oracle(metric):
    dim, nlist, m = 64, 48, 16
    data, cent, books, list_of, codes = _build(12000, dim, nlist, m, 1, metric)
    queries = data[::97][:80] + np.float32(0.25)
    if metric == pxo.COSINE:
        queries /= np.linalg.norm(queries, axis=1, keepdims=True)
    idx = IvfPqIndex(dim, len(cent), m, Metric(metric)).from_parts(cent, books)
    idx.set_store(data)
    idx.set_codes(list_of, codes)
    for nprobe in (1, 4, 16, 100):
        for rerank in (0, 40):
            ref = pxo.ivfpq_search(data, cent, books, m, list_of, codes, queries, 10, nprobe, rerank=rerank,
                                   metric=metric)
            got = idx.search_batch(queries, 10, nprobe, rerank)
            _same(got, ref, f"metric {metric} nprobe {nprobe} rerank {rerank}")


def test_ids_dead_slots_filter_and_large_k():
    dim, nlist, m = 64, 32, 8
    data, cent, books, list_of, codes = _build(9000, dim, nlist, m, 2)
    rng = np.random.default_rng(5)
    ids = rng.permutation(np.arange(10**12, 10**12 + 9000, dtype=np.uint64))
    live = (rng.random(9000) > 0.1).astype(np.uint8)
    bitmap = np.zeros((9000 + 63) // 64, dtype=np.uint64)
    keep = np.flatnonzero(rng.random(9000) > 0.3)
    for s in keep:
        bitmap[s >> 6] |= np.uint64(1) << np.uint64(s & 63)
    queries = data[5::151][:40] + np.float32(1.0)
    idx = IvfPqIndex(dim, nlist, m).from_parts(cent, books)
    idx.set_store(data, ids=ids, live=live)
    idx.set_codes(list_of, codes)
    for k, nprobe, rerank, bm in [(10, 6, 0, None), (10, 6, 30, bitmap), (200, 10, 300, None), (300, 32, 0, bitmap)]:
        ref = pxo.ivfpq_search(data, cent, books, m, list_of, codes, queries, k, nprobe, rerank=rerank, ids=ids,
                               live=live, bitmap=bm)
        got = idx.search_batch(queries, k, nprobe, rerank, bitmap=bm)
        _same(got, ref, f"k {k} nprobe {nprobe} rerank {rerank} filtered {bm is not None}")


def test_uneven_subspace_widths_and_tails():
    dim, nlist, m = 100, 20, 12  # widths 9 x 4 and 8 x 8; dim % 8 == 4
    data, cent, books, list_of, codes = _build(5000, dim, nlist, m, 3)
    queries = data[::123][:30] + np.float32(0.5)
    idx = IvfPqIndex(dim, nlist, m).from_parts(cent, books)
    idx.set_store(data)
    idx.set_codes(list_of, codes)
    for nprobe, rerank in [(3, 0), (7, 25)]:
        ref = pxo.ivfpq_search(data, cent, books, m, list_of, codes, queries, 10, nprobe, rerank=rerank)
        got = idx.search_batch(queries, 10, nprobe, rerank)
        _same(got, ref, f"nprobe {nprobe} rerank {rerank}")


def test_degenerate_calls():
    dim, nlist, m = 32, 8, 4
    data, cent, books, list_of, codes = _build(2000, dim, nlist, m, 4)
    idx = IvfPqIndex(dim, nlist, m).from_parts(cent, books)
    idx.set_store(data)
    idx.set_codes(list_of, codes)
    q = data[:5]
    _, _, lens = idx.search_batch(q, 0, 4)
    assert not lens.any()
    ref = pxo.ivfpq_search(data, cent, books, m, list_of, codes, q, 10, 0)
    _same(idx.search_batch(q, 10, 0), ref, "nprobe 0 clamps to 1")
    ref = pxo.ivfpq_search(data, cent, books, m, list_of, codes, q, 10, 99)
    _same(idx.search_batch(q, 10, 99), ref, "nprobe clamps to nlist")


def test_u8_rerank_integer_rows_and_mixed_queries():
    """Integer rows in [0,255]: the re-rank reads u8 rows for integer queries and f32 rows for the
    others (one batch holds both); a store with one non-integer row re-ranks in f32 throughout."""
    dim, nlist, m = 128, 40, 16
    data, cent, books, list_of, codes = _build(15000, dim, nlist, m, 7)
    queries = np.concatenate([data[3::301][:40],
                              fixtures.blobs_u8(40, dim, 64, fixtures.C4_CENTRES + 7, fixtures.C4_QUERIES),
                              data[7::409][:20] + np.float32(0.5)])
    queries[5, 17] = 256.0  # an integer outside [0,255]
    rng = np.random.default_rng(8)
    ids = rng.permutation(np.arange(5, 5 + 15000, dtype=np.uint64) * 3)
    live = (rng.random(15000) > 0.08).astype(np.uint8)
    bitmap = np.zeros((15000 + 63) // 64, dtype=np.uint64)
    for s_ in np.flatnonzero(rng.random(15000) > 0.4):
        bitmap[s_ >> 6] |= np.uint64(1) << np.uint64(s_ & 63)
    for rows in (data, np.where(np.arange(15000)[:, None] == 77, data + np.float32(0.5), data)):
        idx = IvfPqIndex(dim, nlist, m).from_parts(cent, books)
        idx.set_store(rows, ids=ids, live=live)
        idx.set_codes(list_of, codes)
        for k, nprobe, rerank, bm in [(10, 8, 200, None), (10, 40, 1000, bitmap), (50, 5, 60, None)]:
            ref = pxo.ivfpq_search(rows, cent, books, m, list_of, codes, queries, k, nprobe, rerank=rerank, ids=ids,
                                   live=live, bitmap=bm)
            got = idx.search_batch(queries, k, nprobe, rerank, bitmap=bm)
            _same(got, ref, f"k {k} nprobe {nprobe} rerank {rerank} filtered {bm is not None}")


def test_encode_all_matches_oracle():
    dim, nlist, m = 64, 300, 16  # nlist >= 256: the coarse assignment takes the tensor-core screen
    data, cent, books, list_of, codes = _build(20000, dim, nlist, m, 5)
    rng = np.random.default_rng(2)
    live = (rng.random(len(data)) > 0.05).astype(np.uint8)
    idx = IvfPqIndex(dim, len(cent), m).from_parts(cent, books)
    idx.set_store(data, live=live)
    idx.encode_all()
    _, _, g_list, g_codes = idx.parts()
    r_list = np.zeros(len(data), np.uint32)
    r_codes = np.zeros((len(data), m), np.uint8)
    from oracle.pxo import lib, _p
    lib().pxo_ivfpq_encode_all(_p(data), _p(live), len(data), dim, _p(cent), len(cent), _p(books), m,
                               _p(r_list), _p(r_codes), 8)
    assert np.array_equal(g_list, r_list)
    assert np.array_equal(g_codes[live == 1], r_codes[live == 1])
    queries = data[::211][:30]
    ref = pxo.ivfpq_search(data, cent, books, m, r_list, r_codes, queries, 10, 8, rerank=20, live=live)
    _same(idx.search_batch(queries, 10, 8, 20), ref, "search after a device encode")


@pytest.mark.parametrize("nlist", [40, 300])
def test_train_matches_oracle(nlist):
    dim, m = 32, 8
    data = fixtures.blobs_u8(12000, dim, 80, fixtures.C4_CENTRES + 9, fixtures.C4_BASE + 9)
    cent, books, list_of, codes, rep = pxo.ivfpq_train(data, nlist, m, max_iterations=6, training_sample=3000,
                                                       seed=0x1FF9C0D)
    idx = IvfPqIndex(dim, nlist, m)
    idx.set_store(data)
    got = idx.train(training_sample=3000, max_iterations=6, seed=0x1FF9C0D)
    g_cent, g_books, g_list, g_codes = idx.parts()
    assert got["sampled"] == rep.sampled and got["produced"] == len(cent)
    assert np.array_equal(g_cent.view(np.uint32), cent.view(np.uint32))
    assert np.array_equal(g_books.view(np.uint32), books.view(np.uint32))
    assert np.array_equal(g_list, list_of) and np.array_equal(g_codes, codes)
    assert got["coarse_iterations"] == rep.coarse_iterations
    assert got["coarse_inertia"] == rep.coarse_inertia and got["residual_inertia"] == rep.residual_inertia
    assert got["populated_lists"] == rep.populated_lists and got["largest_list"] == rep.largest_list
