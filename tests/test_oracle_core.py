"""Pin the CPU oracle against the reference's own known-answer tests (distance, space, TopK, flat).

The reference is Rust and cannot be built here; tests/golden/reference_kat.json
transcribes the constants of its unit tests, each with its file:line.
"""
import json
import math
from pathlib import Path

import numpy as np
import pytest

from oracle import pxo

KAT = json.loads((Path(__file__).parent / "golden" / "reference_kat.json").read_text())


def test_distance_known_values():
    k = KAT["distance_known_values"]
    assert pxo.squared_euclidean(k["a"], k["b"]) == k["squared_euclidean"]
    assert math.sqrt(pxo.squared_euclidean(k["a"], k["b"])) == k["euclidean"]
    assert pxo.manhattan(k["a"], k["b"]) == k["manhattan"]
    assert pxo.dot(k["a"], k["b"]) == k["dot"]
    assert pxo.space_distance(pxo.INNER_PRODUCT, k["a"], k["b"]) == k["inner_product"]


def test_cosine_cases_and_zero_vector():
    c = KAT["cosine_cases"]
    for a, b, want in c["cases"]:
        assert abs(pxo.cosine(a, b) - want) < c["tolerance"]
    z = KAT["cosine_zero_vector"]
    assert pxo.cosine(z["a"], z["b"]) == z["value"]


def test_cosine_unit_fast_path():
    c = KAT["cosine_unit_fast_path"]
    a, b = pxo.normalized(c["a"]), pxo.normalized(c["b"])
    assert abs(pxo.cosine(a, b) - pxo.cosine_normalized(a, b)) < c["tolerance"]


def test_tail_lengths_agree_with_scalar():
    t = KAT["tail_lengths"]
    for dim in range(0, t["max_dim"] + 1):
        a = np.array([i * 0.5 - 3.0 for i in range(dim)], dtype=np.float32)
        b = np.array([7.0 - i * 0.25 for i in range(dim)], dtype=np.float32)
        s = pxo.squared_euclidean_scalar(a, b)
        u = pxo.squared_euclidean(a, b)
        assert abs(s - u) <= t["rel_tol"] * max(abs(s), 1.0), dim


def test_exact_symmetry_of_l2_and_dot():
    # crates/proxima-core/tests/metric_properties.rs:108-117: symmetry is exact.
    rng = np.random.default_rng(1)
    for dim in (1, 7, 8, 33, 128):
        a, b = rng.standard_normal(dim).astype(np.float32), rng.standard_normal(dim).astype(np.float32)
        assert pxo.squared_euclidean(a, b) == pxo.squared_euclidean(b, a)
        assert pxo.dot(a, b) == pxo.dot(b, a)
        assert pxo.manhattan(a, b) == pxo.manhattan(b, a)


def test_normalize_and_prepare():
    n = KAT["normalize"]
    v = np.array(n["v"], dtype=np.float32)
    out = pxo.normalized(v)
    assert abs(math.sqrt(pxo.dot(out, out)) - 1.0) < 1e-6
    z = pxo.normalized([0.0, 0.0])
    assert list(z) == [0.0, 0.0]
    p = KAT["prepared_cosine_matches_general"]
    a, b = pxo.prepare(pxo.COSINE, p["a"])[0], pxo.prepare(pxo.COSINE, p["b"])[0]
    assert abs(pxo.space_distance(pxo.COSINE, a, b) - pxo.cosine(p["a"], p["b"])) < p["tolerance"]


def test_host_prepare_matches_oracle_bit_for_bit():
    """proxima_b200.core.prepare_batch (numpy, the host side) == oracle prepare."""
    from proxima_b200.core import Metric, VectorSpace

    rng = np.random.default_rng(7)
    for dim in (5, 8, 64, 100):
        rows = rng.standard_normal((50, dim)).astype(np.float32) * 3
        rows[3] = 0.0
        mine = VectorSpace(dim, Metric.COSINE).prepare_batch(rows)
        ref = pxo.prepare(pxo.COSINE, rows)
        assert np.array_equal(mine.view(np.uint32), ref.view(np.uint32))


def _flat(rows, ids, queries, k, metric=pxo.EUCLIDEAN, bitmap=None, live=None):
    return pxo.flat_search(np.asarray(rows, np.float32), np.asarray(queries, np.float32), k, metric,
                           ids=np.asarray(ids, np.uint64), live=live, bitmap=bitmap)


def test_flat_ties_break_on_id():
    t = KAT["flat_ties"]
    rows = [t["vector"]] * len(t["insert_ids"])
    ids, _, lens = _flat(rows, t["insert_ids"], [t["vector"]], t["k"])
    assert list(ids[0, : lens[0]]) == t["expected_ids"]


def test_flat_filter_runs_during_scan():
    f = KAT["flat_filter"]
    rows = [[float(i)] for i in range(f["n"])]
    keep = np.array([i % f["keep_every"] == 0 for i in range(f["n"])])
    bitmap = np.packbits(keep, bitorder="little")
    bitmap = np.concatenate([bitmap, np.zeros(-len(bitmap) % 8, np.uint8)]).view(np.uint64)
    ids, _, lens = _flat(rows, list(range(f["n"])), [[0.0]], f["k"], bitmap=bitmap)
    assert list(ids[0, : lens[0]]) == f["expected_ids"]


def test_flat_k_larger_and_k_zero_and_empty():
    g = KAT["flat_k_larger_than_index"]
    rows = [[float(i)] for i in range(g["n"])]
    _, _, lens = _flat(rows, list(range(g["n"])), [[0.0]], g["k"])
    assert lens[0] == g["expected_len"]
    _, _, lens = _flat(rows, list(range(g["n"])), [[0.0]], 0)
    assert lens[0] == 0


def test_flat_try_from():
    t = KAT["flat_try_from"]
    rows = np.array(t["data"], np.float32).reshape(-1, 2)
    ids, _, _ = _flat(rows, list(range(3)), [t["query"]], 1)
    assert ids[0, 0] == t["expected_id"]


def test_total_order_nan_and_negative_zero():
    # topk.rs:63-67 uses total_cmp: -0.0 < +0.0 and NaN sorts last.
    rows = np.array([[0.0], [1.0]], np.float32)
    ids, d, _ = pxo.flat_search(rows, np.array([[0.0]], np.float32), 2, pxo.INNER_PRODUCT,
                                ids=np.array([5, 3], np.uint64))
    # dot with 0 query is +0.0 for both; IP = -0.0; tie -> smaller id first
    assert list(ids[0]) == [3, 5]
    assert np.signbit(d[0, 0])


def test_recall_overlap():
    e = np.array([1, 2, 3, 4], np.uint64)
    a = np.array([2, 9, 4], np.uint64)
    assert pxo.lib().pxo_recall_overlap(e.ctypes.data, 4, a.ctypes.data, 3) == 0.5
    assert pxo.lib().pxo_recall_overlap(e.ctypes.data, 0, a.ctypes.data, 3) == 1.0


def _grouped_search(data, ids, queries, k, ngroups, group_k=32):
    """The decomposition the device uses for 32 < k <= 128, restated on the oracle: each
    contiguous group's own top group_k, merged by (distance, id), and the per-query check
    that every full group list ends at or behind the merged k-th entry."""
    bounds = np.linspace(0, len(data), ngroups + 1).astype(int)
    lists = [pxo.flat_search(data[a:b], queries, group_k, pxo.EUCLIDEAN, ids=ids[a:b])
             for a, b in zip(bounds[:-1], bounds[1:])]
    merged, proven = [], []
    for q in range(len(queries)):
        cand = []
        for gi, gd, gl in lists:
            cand += [(float(gd[q, i]), int(gi[q, i])) for i in range(int(gl[q]))]
        cand.sort()
        top = cand[:k]
        ok = True
        for gi, gd, gl in lists:
            if int(gl[q]) < group_k:
                continue
            last = (float(gd[q, group_k - 1]), int(gi[q, group_k - 1]))
            if len(top) < k or last < top[-1]:
                ok = False
        merged.append(top)
        proven.append(ok)
    return merged, proven


def test_grouped_top_k_is_exact_whenever_the_check_passes():
    rng = np.random.default_rng(21)
    centres = rng.integers(0, 256, (40, 16))
    rows = np.clip(np.rint(centres[np.arange(6000) % 40] + rng.normal(0, 12, (6000, 16))), 0, 255)
    rows = rows.astype(np.float32)
    rows[3000:3045] = rows[10]  # 45 copies in one group: the queries near row 10 cannot be proven
    ids = rng.permutation(np.arange(100, 6100, dtype=np.uint64))
    queries = np.concatenate([rows[10:11], rows[::97][:60] + 1.0]).astype(np.float32)
    k = 100
    merged, proven = _grouped_search(rows, ids, queries, k, 8)
    full_i, full_d, full_l = pxo.flat_search(rows, queries, k, pxo.EUCLIDEAN, ids=ids)
    assert not proven[0]
    assert sum(proven) >= 50
    for q in range(len(queries)):
        exact = [(float(full_d[q, i]), int(full_i[q, i])) for i in range(int(full_l[q]))]
        if proven[q]:
            assert merged[q] == exact
    # the failing query really differs: the group kept only 32 of the 45 copies
    exact0 = [(float(full_d[0, i]), int(full_i[0, i])) for i in range(int(full_l[0]))]
    assert merged[0] != exact0


@pytest.mark.parametrize("dim", [1, 7, 16, 100, 128, 255, 256])
def test_integer_vectors_have_exact_f32_squared_euclidean(dim):
    """The premise of the u8 scans (flat K1, the IVF-PQ u8 re-rank): for integer components in
    [0,255] and dim <= 256 the reference's 8-lane f32 squared_euclidean equals the exact integer
    sum, the extreme pair (all 0 against all 255) included."""
    rng = np.random.default_rng(dim)
    pairs = [(np.zeros(dim), np.full(dim, 255.0)), (np.full(dim, 255.0), np.zeros(dim))]
    pairs += [(rng.integers(0, 256, dim).astype(np.float64), rng.integers(0, 256, dim).astype(np.float64))
              for _ in range(200)]
    for a, b in pairs:
        exact = int(((a.astype(np.int64) - b.astype(np.int64)) ** 2).sum())
        assert exact < 2 ** 24
        got = pxo.squared_euclidean(a.astype(np.float32), b.astype(np.float32))
        assert got == float(exact)


def _two_squares(d: float) -> list[float]:
    """An integer point (a, b) with a^2 + b^2 == d: its squared distance to the origin is d exactly."""
    n = int(d)
    for a in range(int(math.isqrt(n)) + 1):
        b = math.isqrt(n - a * a)
        if a * a + b * b == n:
            return [float(a), float(b)]
    raise ValueError(d)


def test_topk_known_answers_through_the_flat_scan():
    """TopK's own tests (topk.rs:215-265), replayed as slots of a flat scan from the origin."""
    t = KAT["topk_best_k"]
    ids = [i for i, _ in t["pushes"]]
    rows = [_two_squares(d) for _, d in t["pushes"]]
    got, dist, lens = _flat(rows, ids, [[0.0, 0.0]], t["k"])
    assert list(got[0, : lens[0]]) == t["expected_ids"]
    assert list(dist[0, : lens[0]]) == sorted(d for _, d in t["pushes"])[: t["k"]]
    # ties break on id whatever the slot (arrival) order
    t = KAT["topk_ties"]
    answers = []
    for order in t["orders"]:
        rows = [_two_squares(t["distance"])] * len(order)
        got, _, lens = _flat(rows, order, [[0.0, 0.0]], t["k"])
        answers.append(list(got[0, : lens[0]]))
    assert answers[0] == answers[1] == sorted(t["orders"][0])[: t["k"]]
    # k = 0 returns nothing; fewer candidates than k is not an error
    t = KAT["topk_k_zero_and_short"]
    _, _, lens = _flat([[1.0, 0.0]], [1], [[0.0, 0.0]], 0)
    assert int(lens[0]) == t["k_zero_len"]
    _, _, lens = _flat([[1.0, 0.0]] * t["short_pushes"], list(range(1, t["short_pushes"] + 1)), [[0.0, 0.0]],
                       t["short_k"])
    assert int(lens[0]) == t["short_len"]
