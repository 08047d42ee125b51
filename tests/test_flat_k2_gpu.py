"""The tensor-core path for non-integer data (K2: f16 screen, exact re-rank,
per-query proof) against the oracle's FlatIndex::search
(crates/proxima-index/src/flat.rs:153-169), bit for bit: identical ids in
identical order and identical f32 distances, for every query, including the
queries the screen could not prove (those run on the fp32 scan).
"""
import numpy as np
import pytest

from oracle import pxo
from proxima_b200 import fixtures
from proxima_b200.core import Metric, VectorSpace
from proxima_b200.index import FlatIndex

pytestmark = pytest.mark.gpu


def _check(data, queries, k, metric, ids=None, expect_path=2, max_redo=None):
    space = VectorSpace(data.shape[1], metric)
    if ids is None:
        ids = np.arange(len(data), dtype=np.uint64)
        idx = FlatIndex.from_array(space, data)
    else:
        idx = FlatIndex(space, capacity=len(data))
        for i, v in zip(ids.tolist(), data):
            idx.insert(int(i), v)
    assert idx.device_path() == expect_path
    pq = space.prepare_batch(queries)
    gi, gd, gl = idx.search_prepared_batch(pq, k)
    prepared = space.prepare_batch(data)
    slot_ids = np.asarray(ids, np.uint64)
    ri, rd, rl = pxo.flat_search(prepared, pq, k, int(metric), ids=slot_ids)
    assert np.array_equal(gl, rl), "lengths"
    for q in range(len(pq)):
        n = int(rl[q])
        assert np.array_equal(gi[q, :n], ri[q, :n]), f"query {q}: ids {gi[q, :n]} vs {ri[q, :n]}"
        assert np.array_equal(gd[q, :n].view(np.uint32), rd[q, :n].view(np.uint32)), f"query {q}: distances"
    redo = idx.last_redone()
    if max_redo is not None:
        assert redo <= max_redo, f"{redo} of {len(pq)} queries were not proven by the screen"
    idx.close()
    return redo


def test_c1_quickstart_cosine():
    """The reference's quickstart (examples/quickstart.rs): 5,000 x 64 cosine,
    queries every 50th vector. Near-duplicate rows (id % 50 classes) make many
    queries unprovable by the screen; they must still come back exact."""
    data = fixtures.quickstart(5000, 64)
    _check(data, data[::50], 10, Metric.COSINE)


@pytest.mark.parametrize("metric", [Metric.EUCLIDEAN, Metric.COSINE, Metric.INNER_PRODUCT])
def test_real_valued_blobs(metric):
    data = fixtures.blobs_f32(120_000, 128, 1024, fixtures.C2_CENTRES, fixtures.C2_BASE)
    queries = fixtures.blobs_f32(1500, 128, 1024, fixtures.C2_CENTRES, fixtures.C2_QUERIES)
    redo = _check(data, queries, 10, metric)
    assert redo < len(queries) // 4, redo


@pytest.mark.parametrize("k", [1, 7, 24])
def test_sphere_blobs_cosine_k(k):
    data = fixtures.sphere_blobs(60_000, 96, 500, fixtures.C5_CENTRES, fixtures.C5_BASE, 0.05)
    queries = fixtures.sphere_blobs(700, 96, 500, fixtures.C5_CENTRES, fixtures.C5_QUERIES, 0.05)
    _check(data, queries, k, Metric.COSINE)


@pytest.mark.parametrize("dim", [1, 7, 33, 64, 100, 128])
def test_dims(dim):
    rng = np.random.default_rng(dim)
    data = (rng.standard_normal((9000, dim)) * 3 + 1).astype(np.float32)
    queries = (rng.standard_normal((300, dim)) * 3 + 1).astype(np.float32)
    _check(data, queries, 10, Metric.EUCLIDEAN)


def test_ties_duplicates_and_shuffled_ids():
    """Duplicate rows under shuffled ids: equal exact distances order by id."""
    rng = np.random.default_rng(5)
    base = (rng.standard_normal((3000, 48)) * 0.5).astype(np.float32)
    data = np.concatenate([base, base, base[:1000]])  # every row two or three times
    ids = rng.permutation(np.arange(10_000, 10_000 + len(data))).astype(np.uint64)
    queries = np.concatenate([base[:200], (rng.standard_normal((100, 48)) * 0.5).astype(np.float32)])
    _check(data, queries, 5, Metric.EUCLIDEAN, ids=ids)
    _check(data, queries, 5, Metric.INNER_PRODUCT, ids=ids)


def test_small_stores_and_k_beyond_the_screen():
    rng = np.random.default_rng(9)
    for n in (1, 5, 31, 32, 33, 300):
        data = rng.standard_normal((n, 16)).astype(np.float32)
        queries = rng.standard_normal((40, 16)).astype(np.float32)
        _check(data, queries, 10, Metric.EUCLIDEAN)
    data = rng.standard_normal((5000, 16)).astype(np.float32)
    queries = rng.standard_normal((50, 16)).astype(np.float32)
    _check(data, queries, 25, Metric.EUCLIDEAN)  # k > 24: the fp32 scan (same answer)


def test_wide_dynamic_range():
    """Rows far from the origin (large mean) and tiny spreads: the centring and
    the power-of-two scales keep the screen's bound meaningful."""
    rng = np.random.default_rng(11)
    data = (1e4 + rng.standard_normal((20_000, 32)) * 1e-2).astype(np.float32)
    queries = (1e4 + rng.standard_normal((200, 32)) * 1e-2).astype(np.float32)
    _check(data, queries, 10, Metric.EUCLIDEAN)
    small = (rng.standard_normal((20_000, 32)) * 1e-8).astype(np.float32)
    _check(small, small[:100] * 1.5, 10, Metric.EUCLIDEAN)


def test_filtered_and_manhattan_searches_stay_on_the_fp32_scan():
    rng = np.random.default_rng(13)
    data = rng.standard_normal((4000, 24)).astype(np.float32)
    space = VectorSpace(24, Metric.MANHATTAN)
    idx = FlatIndex.from_array(space, data)
    assert idx.device_path() == 0
    idx.close()
    space = VectorSpace(24, Metric.EUCLIDEAN)
    idx = FlatIndex.from_array(space, data)
    assert idx.device_path() == 2
    hits = idx.search(data[7], 5, lambda i, m: i % 3 == 0)
    bits = np.packbits((np.arange(4000) % 3 == 0).astype(np.uint8), bitorder="little")
    bitmap = np.pad(bits, (0, 504 - bits.size)).view(np.uint64)
    ri, rd, rl = pxo.flat_search(data, data[7:8], 5, pxo.EUCLIDEAN, bitmap=bitmap)
    assert [h.id for h in hits] == [int(x) for x in ri[0, :rl[0]]]
    idx.close()


def test_unproven_queries_take_the_range_scan_and_its_overflow():
    """5,000 copies of one row: a query equal to it ties with all of them, the
    screen cannot prove it, and the exact range scan collects more rows than
    its capacity (4,096), so the query ends on the fp32 scan; a query at a
    small offset is proven or range-scanned. Answers order the ties by id."""
    rng = np.random.default_rng(17)
    dup = rng.standard_normal(16).astype(np.float32)
    data = np.concatenate([np.tile(dup, (5000, 1)), rng.standard_normal((3000, 16)).astype(np.float32)])
    ids = rng.permutation(len(data)).astype(np.uint64)
    queries = np.stack([dup, dup + np.float32(0.01), rng.standard_normal(16).astype(np.float32)])
    redo = _check(data, queries, 10, Metric.EUCLIDEAN, ids=ids)
    assert redo >= 1
