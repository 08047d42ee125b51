"""Scalar quantization on the GPU (pxc_sq_*) against the oracle.

ScalarQuantizer::train / encode_into / decode (crates/proxima-quantize/src/scalar.rs:141-296)
bit for bit, including the reference's own known answers (scalar.rs:365-451),
the sign of a zero bound and NaN / out-of-range clamping; and the filtered
search (int8 over-fetch on tcgen05, exact re-rank) against the oracle's
restatement of the same composition: ids, distances and lengths bit for bit,
for both metrics, every filter form, ragged dimensions, dead slots, VectorIds
that are not slot numbers, ties, empty results and the exact fallback. On
separated data its top-k equals the exact filtered FlatIndex answer."""
import json
import os
from pathlib import Path

import numpy as np
import pytest

from oracle import pxo
from proxima_b200 import fixtures
from proxima_b200.core import Metric
from proxima_b200.sq import CodeType, IntRange, RangeMode, ScalarQuantizer, SqIndex, combine_ranges

pytestmark = pytest.mark.gpu

KAT = json.loads((Path(__file__).parent / "golden" / "reference_kat.json").read_text())


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def _train_both(t, dim, mode):
    sq = ScalarQuantizer.train(dim, t, mode)
    mn, sc, inv = pxo.sq_train(np.asarray(t, np.float32).reshape(-1, dim), int(mode))
    return sq, (mn, sc, inv)


def test_known_answers():
    c = KAT["sq_clamp"]
    sq = ScalarQuantizer.train(1, np.array(c["training"], np.float32), RangeMode.PER_DIMENSION)
    lo = sq.decode(sq.encode(np.array([c["low"]], np.float32)))
    hi = sq.decode(sq.encode(np.array([c["high"]], np.float32)))
    assert lo[0, 0] == c["low_decoded"] and hi[0, 0] == c["high_decoded"]
    k = KAT["sq_constant_dim"]
    sq = ScalarQuantizer.train(2, np.array(k["training"], np.float32), RangeMode.PER_DIMENSION)
    assert sq.scale[0] == 0.0 and sq.inverse_scale[0] == 0.0
    dec = sq.decode(sq.encode(np.array(k["probe"], np.float32)))
    assert dec[0, 0] == k["decoded0"]
    # half-step bound and identical U8 / I8 lattices (scalar.rs:365-427)
    t = np.array([[i / 255.0, 1000.0 * i / 255.0] for i in range(256)], np.float32)
    u8 = ScalarQuantizer.train(2, t, RangeMode.PER_DIMENSION, CodeType.U8)
    i8 = ScalarQuantizer.train(2, t, RangeMode.PER_DIMENSION, CodeType.I8)
    du = u8.decode(u8.encode(t))
    di = i8.decode(i8.encode(t))
    assert np.all(np.abs(du[:, 0] - t[:, 0]) <= (1 / 255) / 2 + 1e-5)
    assert np.all(np.abs(du[:, 1] - t[:, 1]) <= (1000 / 255) / 2 + 1e-5)
    assert np.array_equal(du, di)


@pytest.mark.parametrize("mode", [RangeMode.PER_DIMENSION, RangeMode.GLOBAL])
@pytest.mark.parametrize("dim", [1, 7, 64, 100, 768])
def test_train_encode_decode_match_oracle(mode, dim):
    rng = np.random.default_rng(dim * 7 + int(mode))
    n = 3000
    t = (rng.standard_normal((n, dim)) * rng.uniform(0.1, 5.0, dim)).astype(np.float32)
    # zeros of both signs, first a -0 then a +0 in some columns, the reverse in others
    t[:, : max(1, dim // 3)] = np.abs(t[:, : max(1, dim // 3)])
    t[5, : max(1, dim // 3)] = -0.0
    t[9, : max(1, dim // 3)] = 0.0
    t[2, : max(1, dim // 6)] = 0.0
    sq, (mn, sc, inv) = _train_both(t, dim, mode)
    assert np.array_equal(_bits(sq.min), _bits(mn))
    assert np.array_equal(_bits(sq.scale), _bits(sc))
    assert np.array_equal(_bits(sq.inverse_scale), _bits(inv))
    # encode: in-range, out-of-range, NaN and infinities
    probe = np.concatenate([t[:500], (rng.standard_normal((300, dim)) * 20).astype(np.float32)])
    probe[3, 0] = np.nan
    probe[4, 0] = np.inf
    probe[6, 0] = -np.inf
    for ct in (CodeType.U8, CodeType.I8):
        q = ScalarQuantizer(dim, mode, ct, sq.min, sq.scale, sq.inverse_scale)
        got = q.encode(probe)
        ref = pxo.sq_encode(mn, inv, dim, int(mode), int(ct), probe)
        assert np.array_equal(got, ref), f"codes differ ({ct.name})"
        dec = q.decode(got)
        assert np.array_equal(_bits(dec), _bits(pxo.sq_decode(mn, sc, dim, int(mode), int(ct), ref)))


def test_train_device_and_sharded_ranges():
    import torch

    from proxima_b200.sq import ranges_device

    rng = np.random.default_rng(3)
    dim = 96
    t = rng.standard_normal((20000, dim)).astype(np.float32)
    t[:, 0] = np.abs(t[:, 0])
    t[7000, 0] = -0.0  # first zero sits in the second shard
    t[15000, 0] = 0.0
    mn, sc, inv = pxo.sq_train(t, pxo.RANGE_PER_DIMENSION)
    dev = torch.from_numpy(t).cuda()
    sq = ScalarQuantizer.train(dim, dev, RangeMode.PER_DIMENSION)
    assert np.array_equal(_bits(sq.min), _bits(mn)) and np.array_equal(_bits(sq.inverse_scale), _bits(inv))
    codes = sq.encode(dev).cpu().numpy()
    assert np.array_equal(codes, pxo.sq_encode(mn, inv, dim, 1, 0, t))
    # per-shard ranges folded in shard order == the single pass
    lows, highs = [], []
    for a, b in ((0, 5000), (5000, 12000), (12000, 20000)):
        lo, hi = ranges_device(dev[a:b], dim)
        lows.append(lo)
        highs.append(hi)
    cmn, csc, cinv = combine_ranges(lows, highs)
    assert np.array_equal(_bits(cmn), _bits(mn)) and np.array_equal(_bits(csc), _bits(sc))
    assert np.array_equal(_bits(cinv), _bits(inv))


def test_train_errors():
    from proxima_b200.errors import Configuration, NonFinite

    t = np.ones((4, 3), np.float32)
    t[2, 1] = np.nan
    with pytest.raises(NonFinite) as e:
        ScalarQuantizer.train(3, t)
    assert e.value.index == 1
    with pytest.raises(Configuration):
        ScalarQuantizer.train(3, np.zeros(0, np.float32))


# ---------------------------------------------------------------------------
# filtered search
# ---------------------------------------------------------------------------
def _corpus(n, dim, nblobs, seed, sigma=0.03):
    data = fixtures.sphere_blobs(n, dim, nblobs, fixtures.C5_CENTRES + seed, fixtures.C5_BASE + seed, sigma)
    years = fixtures.uniform_int(n, fixtures.C5_YEARS + seed, 2000, 30)
    return data, years


def _oracle_search(sq, data, ids, live, accepted_slot, queries, k, overfetch, metric):
    """The oracle over rank order (ascending id among live slots)."""
    slots = np.nonzero(live)[0] if live is not None else np.arange(len(data))
    order = slots[np.argsort(ids[slots], kind="stable")]
    codes = pxo.sq_encode(sq.min, sq.inverse_scale, data.shape[1], int(sq.mode), pxo.CODE_I8, data[order])
    acc = None if accepted_slot is None else accepted_slot[order].astype(np.uint8)
    return pxo.sq_search(sq.scale, int(sq.mode), codes, data[order], queries, k, overfetch, metric,
                         ids=ids[order], accepted=acc)


def _same(got, ref, label):
    gi, gd, gl = got
    ri, rd, rl = ref
    assert np.array_equal(gl, rl), f"{label}: lengths"
    for q in range(len(rl)):
        n = int(rl[q])
        assert np.array_equal(gi[q, :n], ri[q, :n]), f"{label}: ids of query {q}"
        assert np.array_equal(_bits(gd[q, :n]), _bits(rd[q, :n])), f"{label}: distances of query {q}"


def _bitmap(acc_slot):
    n = len(acc_slot)
    words = np.zeros((n + 63) // 64, np.uint64)
    for s in np.nonzero(acc_slot)[0]:
        words[s >> 6] |= np.uint64(1) << np.uint64(s & 63)
    return words


@pytest.mark.parametrize("metric", [Metric.COSINE, Metric.INNER_PRODUCT])
@pytest.mark.parametrize("dim,n", [(64, 40000), (100, 21000), (37, 3000)])
def test_search_matches_oracle(metric, dim, n):
    data, years = _corpus(n, dim, 200, dim)
    queries = fixtures.sphere_blobs(300, dim, 200, fixtures.C5_CENTRES + dim, fixtures.C5_QUERIES, 0.03)
    ids = np.arange(n, dtype=np.uint64) * 3 + 11
    idx = SqIndex(dim, metric)
    idx.set_store(data, ids=ids)
    sq = idx.train(RangeMode.PER_DIMENSION)
    idx.set_column(0, years)
    k, F = 10, 100
    # no filter, range filter, bitmap, both
    got = idx.search_batch(queries, k, F)
    _same(got, _oracle_search(sq, data, ids, None, None, queries, k, F, int(metric)), "no filter")
    acc_year = years >= 2027
    got = idx.search_batch(queries, k, F, ranges=[IntRange(0, lo=2027)])
    _same(got, _oracle_search(sq, data, ids, None, acc_year, queries, k, F, int(metric)), "year >= 2027")
    assert idx.last_accepted() == int(acc_year.sum())
    acc_bm = (np.arange(n) % 3) != 1
    got = idx.search_batch(queries, k, F, bitmap=_bitmap(acc_bm))
    _same(got, _oracle_search(sq, data, ids, None, acc_bm, queries, k, F, int(metric)), "bitmap")
    both = acc_bm & (years >= 2010) & (years <= 2015)
    got = idx.search_batch(queries, k, F, bitmap=_bitmap(acc_bm), ranges=[IntRange(0, 2010, 2015)])
    _same(got, _oracle_search(sq, data, ids, None, both, queries, k, F, int(metric)), "bitmap + range")


def test_search_global_mode_dead_slots_shuffled_ids():
    dim, n = 96, 30000
    data, years = _corpus(n, dim, 150, 5)
    rng = np.random.default_rng(5)
    ids = rng.permutation(n).astype(np.uint64) * 2
    live = (rng.random(n) > 0.2).astype(np.uint8)
    queries = fixtures.sphere_blobs(200, dim, 150, fixtures.C5_CENTRES + 5, fixtures.C5_QUERIES + 1, 0.03)
    idx = SqIndex(dim, Metric.COSINE)
    idx.set_store(data, ids=ids, live=live)
    sq = idx.train(RangeMode.GLOBAL)
    present = (rng.random(n) > 0.1).astype(np.uint8)
    idx.set_column(3, years, present)
    assert len(idx) == int(live.sum())
    got = idx.search_batch(queries, 25, 300, ranges=[IntRange(3, lo=2020)])
    acc = (years >= 2020) & (present == 1)
    _same(got, _oracle_search(sq, data, ids, live.astype(bool), acc, queries, 25, 300, pxo.COSINE), "global")
    # stored codes are the reference's encode of the live rows
    codes = idx.codes()
    ref = pxo.sq_encode(sq.min, sq.inverse_scale, dim, 0, pxo.CODE_I8, data)
    assert np.array_equal(codes[live == 1], ref[live == 1])


def test_search_forced_fallback_is_identical(monkeypatch):
    dim, n = 64, 50000
    data, years = _corpus(n, dim, 100, 9)
    queries = fixtures.sphere_blobs(150, dim, 100, fixtures.C5_CENTRES + 9, fixtures.C5_QUERIES + 2, 0.03)
    idx = SqIndex(dim, Metric.COSINE)
    idx.set_store(data)
    idx.train()
    idx.set_column(0, years)
    base = idx.search_batch(queries, 10, 100, ranges=[IntRange(0, lo=2003)])
    assert idx.last_fallback() == 0
    idx.ctx.set_option("sq_candidate_cap", 0)
    try:
        forced = idx.search_batch(queries, 10, 100, ranges=[IntRange(0, lo=2003)])
    finally:
        idx.ctx.set_option("sq_candidate_cap", -1)
    assert 0 < idx.last_fallback() <= len(queries)
    _same(forced, base, "fallback")


def test_search_failed_speculation_is_retried_exactly(monkeypatch):
    """With the speculative admission key forced to the best prefix key, most
    queries admit fewer than F rows, fail verification and are scanned again
    with the safe key; the answers do not change."""
    dim, n = 64, 40000
    data, years = _corpus(n, dim, 100, 17)
    queries = fixtures.sphere_blobs(200, dim, 100, fixtures.C5_CENTRES + 17, fixtures.C5_QUERIES + 5, 0.03)
    idx = SqIndex(dim, Metric.COSINE)
    idx.set_store(data)
    sq = idx.train()
    idx.set_column(0, years)
    base = idx.search_batch(queries, 10, 100, ranges=[IntRange(0, lo=2001)])
    idx.ctx.set_option("sq_spec_rank", 1)
    try:
        forced = idx.search_batch(queries, 10, 100, ranges=[IntRange(0, lo=2001)])
    finally:
        idx.ctx.set_option("sq_spec_rank", -1)
    assert idx.last_retried() > len(queries) // 2
    _same(forced, base, "retried")
    acc = years >= 2001
    _same(forced, _oracle_search(sq, data, np.arange(n, dtype=np.uint64), None, acc, queries, 10, 100, pxo.COSINE),
          "retried vs oracle")


def test_ties_empty_and_edges():
    dim = 32
    base = fixtures.sphere_blobs(50, dim, 5, 77, 78, 0.03)
    data = np.repeat(base, 400, axis=0)  # 20000 rows, every row 400 times: equal scores everywhere
    n = len(data)
    ids = np.arange(n, dtype=np.uint64)[::-1].copy()  # ids descending in slot order
    idx = SqIndex(dim, Metric.COSINE)
    idx.set_store(data, ids=ids)
    sq = idx.train()
    idx.set_column(0, np.arange(n, dtype=np.int64))
    q = base[:20]
    for k, F in ((10, 100), (1, 1), (64, 64), (100, 2048)):
        got = idx.search_batch(q, k, F)
        _same(got, _oracle_search(sq, data, ids, None, None, q, k, F, pxo.COSINE), f"ties k={k} F={F}")
    # fewer accepted rows than k; none accepted; k == 0
    got = idx.search_batch(q, 10, 100, ranges=[IntRange(0, 5, 9)])
    assert np.all(got[2] == 5)
    acc = (np.arange(n) >= 5) & (np.arange(n) <= 9)
    _same(got, _oracle_search(sq, data, ids, None, acc, q, 10, 100, pxo.COSINE), "five accepted")
    got = idx.search_batch(q, 10, 100, ranges=[IntRange(0, 10**9)])
    assert np.all(got[2] == 0)
    got = idx.search_batch(q, 0, 100)
    assert np.all(got[2] == 0)


def test_many_queries_span_batches():
    dim, n = 64, 20000
    data, _ = _corpus(n, dim, 80, 13)
    queries = fixtures.sphere_blobs(4500, dim, 80, fixtures.C5_CENTRES + 13, fixtures.C5_QUERIES + 3, 0.03)
    idx = SqIndex(dim, Metric.COSINE)
    idx.set_store(data)
    sq = idx.train()
    got = idx.search_batch(queries, 10, 100)
    ref = _oracle_search(sq, data, np.arange(n, dtype=np.uint64), None, None, queries, 10, 100, pxo.COSINE)
    _same(got, ref, "4500 queries")


def test_top10_equals_exact_filtered_flat():
    """On C5-shaped data the re-ranked top-10 is the exact filtered answer
    (FlatIndex::search with the filter, crates/proxima-index/src/flat.rs:153-169)."""
    dim, n = 768, 60000
    data, years = _corpus(n, dim, 120, 21)
    queries = fixtures.sphere_blobs(64, dim, 120, fixtures.C5_CENTRES + 21, fixtures.C5_QUERIES + 4, 0.03)
    idx = SqIndex(dim, Metric.COSINE)
    idx.set_store(data)
    idx.train()
    idx.set_column(0, years)
    gi, gd, gl = idx.search_batch(queries, 10, 100, ranges=[IntRange(0, lo=2027)])
    acc = years >= 2027
    ri, rd, rl = pxo.flat_search(data, queries, 10, pxo.COSINE, bitmap=_bitmap(acc))
    assert np.array_equal(gl, rl)
    assert np.array_equal(gi, ri)
    assert np.array_equal(_bits(gd), _bits(rd))


def test_row_shards_merge_like_the_per_shard_composition():
    """The C5 multi-GPU form on one GPU: two row shards with global VectorIds, one
    quantizer from the shards' ranges folded in shard order, each shard's exact
    top-k merged on the device (pxc_topk_merge) — equal to the oracle run per
    shard and merged by (total_cmp, id)."""
    import torch

    from proxima_b200 import _native as N
    from proxima_b200.sq import ranges_device

    dim, n, k, F = 64, 30000, 10, 100
    data, years = _corpus(n, dim, 120, 41)
    queries = fixtures.sphere_blobs(120, dim, 120, fixtures.C5_CENTRES + 41, fixtures.C5_QUERIES + 6, 0.03)
    cut = 13000
    parts = [(0, cut), (cut, n)]
    lows, highs = [], []
    for a, b in parts:
        lo, hi = ranges_device(torch.from_numpy(data[a:b]).cuda(), dim)
        lows.append(lo)
        highs.append(hi)
    mn, sc, inv = combine_ranges(lows, highs)
    quant = ScalarQuantizer(dim, RangeMode.PER_DIMENSION, CodeType.I8, mn, sc, inv)
    ref_m, ref_sc, ref_inv = pxo.sq_train(data, pxo.RANGE_PER_DIMENSION)
    assert np.array_equal(_bits(mn), _bits(ref_m)) and np.array_equal(_bits(inv), _bits(ref_inv))
    nq = len(queries)
    g_ids = torch.zeros((2, nq, k), dtype=torch.int64, device="cuda")
    g_d = torch.zeros((2, nq, k), dtype=torch.float32, device="cuda")
    g_l = torch.zeros((2, nq), dtype=torch.int32, device="cuda")
    oracle_parts = []
    for r, (a, b) in enumerate(parts):
        idx = SqIndex(dim, Metric.COSINE)
        ids = np.arange(a, b, dtype=np.uint64)
        idx.set_store(data[a:b], ids=ids)
        idx.set_quantizer(quant)
        idx.set_column(0, years[a:b])
        gi, gd, gl = idx.search_batch(queries, k, F, ranges=[IntRange(0, lo=2025)])
        g_ids[r] = torch.from_numpy(gi.view(np.int64)).cuda()
        g_d[r] = torch.from_numpy(gd).cuda()
        g_l[r] = torch.from_numpy(gl.view(np.int32)).cuda()
        oracle_parts.append(_oracle_search(quant, data[a:b], ids, None, years[a:b] >= 2025, queries, k, F, pxo.COSINE))
        idx.close()
    m_ids = torch.zeros((nq, k), dtype=torch.int64, device="cuda")
    m_d = torch.zeros((nq, k), dtype=torch.float32, device="cuda")
    m_l = torch.zeros(nq, dtype=torch.int32, device="cuda")
    from proxima_b200.index import Context

    ctx = Context.default()
    N.call("pxc_topk_merge", ctx.handle, g_ids.data_ptr(), g_d.data_ptr(), g_l.data_ptr(), 2, nq, k, k,
           m_ids.data_ptr(), m_d.data_ptr(), m_l.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    got = (m_ids.cpu().numpy().view(np.uint64), m_d.cpu().numpy(), m_l.cpu().numpy().view(np.uint32))
    # the oracle's per-shard answers merged by (total_cmp(distance), id)
    ri = np.zeros((nq, k), np.uint64)
    rd = np.zeros((nq, k), np.float32)
    rl = np.zeros(nq, np.uint32)
    def total_key(x):  # f32::total_cmp as a signed integer order
        v = int(np.float32(x).view(np.int32))
        return v ^ ((v >> 31) & 0x7FFFFFFF)

    for q in range(nq):
        cands = [(total_key(pd[q, j]), int(pi[q, j]), pd[q, j]) for pi, pd, pl in oracle_parts
                 for j in range(int(pl[q]))]
        cands.sort(key=lambda c: (c[0], c[1]))
        for j, c in enumerate(cands[:k]):
            ri[q, j], rd[q, j] = c[1], c[2]
        rl[q] = min(k, len(cands))
    _same(got, (ri, rd, rl), "merged shards")
