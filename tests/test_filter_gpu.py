"""Typed filter pushdown on the GPU: MetadataFilter conditions evaluated per
slot over device columns (pxc_columns_eval) equal the oracle's restatement of
filter.rs:216-256 slot for slot, and the filtered flat and IVF-PQ searches that
use them (pxc_flat_search_where, pxc_ivfpq_search_where) equal the oracle's
searches with that accepted set, bit for bit."""
import random

import numpy as np
import pytest
import torch

from oracle import pxo
from proxima_b200 import _native as N
from proxima_b200 import fixtures
from proxima_b200.core import Metric, VectorSpace
from proxima_b200.filters import DeviceColumns, MetadataFilter
from proxima_b200.index import Context, FlatIndex
from proxima_b200.ivfpq import IvfPqIndex
from test_oracle_filter import random_filter, random_metadata

pytestmark = pytest.mark.gpu


def _device_bitmap(cols, flt, nslots):
    conds, nc, ops, no = flt.compile(cols)
    out = torch.zeros((nslots + 63) // 64, dtype=torch.int64, device="cuda")
    N.call("pxc_columns_eval", cols.handle, nslots, conds, nc, ops, no, out.data_ptr(),
           torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return out.cpu().numpy().view(np.uint64)


def test_device_evaluation_equals_the_oracle_slot_by_slot():
    rng = random.Random(3)
    n = 5000
    metas = [random_metadata(rng) for _ in range(n)]
    cols = DeviceColumns(Context.default())
    for field in ("x", "y", "z"):
        cols.set_values(field, [m.get(field) for m in metas])
    for _ in range(200):
        raw = random_filter(rng)
        got = _device_bitmap(cols, MetadataFilter.parse(raw), n)
        want = pxo.slot_bitmap([pxo.metadata_filter_accepts(raw, m) for m in metas])
        assert np.array_equal(got, want), raw
    # slots past a column's end read as absent; a gap before slot_begin too
    cols.set_values("late", [1, 2, 3], slot_begin=100)
    got = _device_bitmap(cols, MetadataFilter.parse({"late": {"exists": True}}), n)
    want = pxo.slot_bitmap([100 <= s < 103 for s in range(n)])
    assert np.array_equal(got, want)
    cols.close()


@pytest.mark.parametrize("integer_rows", [True, False])
def test_flat_search_with_device_filters(integer_rows):
    rng = random.Random(11)
    n, dim = 30_000, 64
    data = fixtures.blobs_u8(n, dim, 128, 7, 8) if integer_rows else fixtures.blobs_f32(n, dim, 128, 7, 8)
    queries = fixtures.blobs_u8(120, dim, 128, 7, 9) if integer_rows else fixtures.blobs_f32(120, dim, 128, 7, 9)
    space = VectorSpace(dim, Metric.EUCLIDEAN)
    idx = FlatIndex(space, capacity=n)
    metas = [random_metadata(rng) for _ in range(n)]
    for i in range(n):
        idx.insert(i, data[i], metas[i])
    for i in range(0, n, 7):  # tombstones: removed ids never come back
        idx.remove(i)
    live = np.ones(n, np.uint8)
    live[::7] = 0
    for _ in range(12):
        raw = random_filter(rng)
        flt = MetadataFilter.parse(raw)
        got = idx.search_batch(queries, 10, flt)
        acc = [bool(live[s]) and pxo.metadata_filter_accepts(raw, metas[s]) for s in range(n)]
        ri, rd, rl = pxo.flat_search(data, queries, 10, pxo.EUCLIDEAN, live=live, bitmap=pxo.slot_bitmap(acc))
        for q in range(len(queries)):
            assert [h.id for h in got[q]] == [int(x) for x in ri[q, :rl[q]]], (raw, q)
            assert np.array_equal(np.array([h.distance for h in got[q]], np.float32).view(np.uint32),
                                  rd[q, :rl[q]].view(np.uint32))
    # metadata changes reach the device columns
    idx.set_metadata(1, {"x": "only"})
    hits = idx.search(data[1], 3, MetadataFilter.parse({"x": "only"}))
    assert [h.id for h in hits] == [1]
    idx.close()


def test_ivfpq_search_with_device_filters():
    rng = random.Random(13)
    n, dim, nlist, m = 20_000, 32, 64, 8
    data = fixtures.blobs_u8(n, dim, 64, 3, 4)
    queries = fixtures.blobs_u8(100, dim, 64, 3, 5)
    cent, books, list_of, codes, _ = pxo.ivfpq_train(data, nlist, m, 4, 10_000, 0x77)
    idx = IvfPqIndex(dim, nlist, m)
    idx.from_parts(cent, books)
    idx.set_store(data)
    idx.set_codes(list_of, codes)
    metas = [random_metadata(rng) for _ in range(n)]
    idx.set_metadata(metas)
    for _ in range(6):
        raw = random_filter(rng)
        gi, gd, gl = idx.search_where(queries, 10, 8, 200, MetadataFilter.parse(raw))
        bm = pxo.slot_bitmap([pxo.metadata_filter_accepts(raw, mm) for mm in metas])
        ri, rd, rl = pxo.ivfpq_search(data, cent, books, m, list_of, codes, queries, 10, 8, 200, bitmap=bm)
        assert np.array_equal(gl, rl), raw
        for q in range(len(queries)):
            assert np.array_equal(gi[q, :rl[q]], ri[q, :rl[q]]), (raw, q)
            assert np.array_equal(gd[q, :rl[q]].view(np.uint32), rd[q, :rl[q]].view(np.uint32)), (raw, q)
    idx.close()
