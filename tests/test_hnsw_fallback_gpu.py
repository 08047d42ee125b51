"""HnswIndex's exhaustive filtered scan (crates/proxima-index/src/hnsw.rs:1189-1198)
on the GPU against the oracle's FlatIndex::search over the same store: detached
(tombstoned) slots are never returned and never reused, highly selective filters
(the case the fallback exists for, hnsw.rs:1129-1140) as host closures and as
device-evaluated MetadataFilters, bit for bit."""
import numpy as np
import pytest

from oracle import pxo
from proxima_b200 import fixtures
from proxima_b200.core import Metric, VectorSpace
from proxima_b200.filters import MetadataFilter
from proxima_b200.hnsw import HnswStoreMirror

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("metric", [Metric.EUCLIDEAN, Metric.COSINE])
def test_exhaustive_fallback_equals_the_oracle(metric):
    n, dim = 20_000, 48
    data = fixtures.blobs_u8(n, dim, 64, 5, 6) if metric == Metric.EUCLIDEAN else \
        fixtures.sphere_blobs(n, dim, 64, 5, 6, 0.1)
    queries = data[::500][:40] + np.float32(0.5 if metric == Metric.EUCLIDEAN else 0.01)
    space = VectorSpace(dim, metric)
    store = HnswStoreMirror(space, capacity=n)
    for i in range(n):
        store.insert(1_000_000 + i, data[i], {"tenant": i % 1000, "tag": "x" if i % 3 else "y"})
    detached = list(range(0, n, 11))
    for i in detached:
        store.remove(1_000_000 + i)
    # a later insert takes a new slot: detached slots are never reused
    store.insert(5, data[0], {"tenant": 7, "tag": "x"})
    assert store._next == n + 1
    rows = np.concatenate([data, data[:1]])
    ids = np.concatenate([np.arange(1_000_000, 1_000_000 + n, dtype=np.uint64), np.array([5], np.uint64)])
    live = np.ones(n + 1, np.uint8)
    live[detached] = 0
    tenant = np.concatenate([np.arange(n) % 1000, [7]])
    prepared = space.prepare_batch(rows)
    pq = space.prepare_batch(queries)
    for flt, acc in ((lambda i, m: m.get("tenant") == 7, tenant == 7),
                     (MetadataFilter.parse({"tenant": {"in": [7, 9]}, "tag": "x"}),
                      ((tenant == 7) | (tenant == 9)) & (np.concatenate([np.arange(n) % 3 != 0, [True]])))):
        got = store.exhaustive_batch(queries, 10, flt)
        ri, rd, rl = pxo.flat_search(prepared, pq, 10, int(metric), ids=ids, live=live,
                                     bitmap=pxo.slot_bitmap(acc & (live == 1)))
        for q in range(len(queries)):
            assert [h.id for h in got[q]] == [int(x) for x in ri[q, :rl[q]]]
            assert np.array_equal(np.array([h.distance for h in got[q]], np.float32).view(np.uint32),
                                  rd[q, :rl[q]].view(np.uint32))
        one = store.exhaustive(queries[3], 10, flt)
        assert [h.id for h in one] == [h.id for h in got[3]]
    store.close()
