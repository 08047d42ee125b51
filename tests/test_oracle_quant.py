"""Pin the oracle's k-means, PQ, SQ and IVF-PQ against the reference's tests.

k-means++ draws depend on rand_chacha / rand, restated from their published
algorithms (parity unpinned); the assertions here are the reference's own,
which hold for any correct k-means++ draw sequence.
"""
import json
from pathlib import Path

import numpy as np
import pytest

from oracle import pxo
from proxima_b200 import fixtures

KAT = json.loads((Path(__file__).parent / "golden" / "reference_kat.json").read_text())


def _blobs():
    b = KAT["kmeans_blobs"]
    pts = []
    for cx, cy in b["centres"]:
        for i in range(b["per_blob"]):
            j = np.float32(i) * np.float32(b["jitter"])
            pts.append([np.float32(cx) + j, np.float32(cy) - j])
    return np.array(pts, np.float32)


def test_kmeans_recovers_blobs():
    b = KAT["kmeans_blobs"]
    cent, _, inertia, _ = pxo.kmeans(_blobs(), b["k"], b["max_iterations"], seed=0x00C0FFEE)
    found = sorted((int(round(c[0])), int(round(c[1]))) for c in cent)
    assert found == [tuple(x) for x in b["expected_rounded"]]
    assert inertia < b["max_inertia"]


def test_kmeans_deterministic_clamp_identical_empty():
    a = pxo.kmeans(_blobs(), 3, 25, seed=0x00C0FFEE)
    b = pxo.kmeans(_blobs(), 3, 25, seed=0x00C0FFEE)
    assert np.array_equal(a[0], b[0]) and a[3] == b[3]
    c = KAT["kmeans_clamp"]
    cent, _, _, _ = pxo.kmeans(np.array(c["points"], np.float32).reshape(-1, c["dim"]), c["k"], 25)
    assert cent.size == c["expected_centroid_floats"]
    i = KAT["kmeans_identical"]
    pts = np.full(i["n_floats"], i["value"], np.float32).reshape(-1, i["dim"])
    cent, _, inertia, _ = pxo.kmeans(pts, i["k"], 25)
    assert inertia == i["inertia"] and np.all(cent == i["value"])


def test_kmeans_inertia_non_increasing():
    prev = np.inf
    for cap in range(1, 8):
        _, _, inertia, _ = pxo.kmeans(_blobs(), 3, cap, seed=0x00C0FFEE)
        assert inertia <= prev + 1e-9
        prev = inertia


def test_kmeans_from_init_matches_a_plain_lloyd():
    """Injected-init Lloyd (the parity mode for config C3) against a direct restatement."""
    rng = np.random.default_rng(3)
    pts = rng.standard_normal((400, 6)).astype(np.float32)
    init = pts[rng.choice(400, 12, replace=False)].copy()
    cent, assign, inertia, iters = pxo.kmeans(pts, 12, 5, init=init)
    c = init.copy()
    a = np.zeros(400, np.uint32)
    for it in range(5):
        d = np.array([[pxo.squared_euclidean_scalar(p, q) for q in c] for p in pts], np.float32)
        best = d.argmin(axis=1).astype(np.uint32)  # argmin takes the first minimum, as strict '<'
        changed = np.any(best != a)
        a = best
        if not changed and it > 0:
            break
        for j in range(12):
            m = a == j
            if m.any():
                s = pts[m].astype(np.float64).sum(axis=0, dtype=np.float64)
                c[j] = (s * (1.0 / m.sum())).astype(np.float32)
    assert np.array_equal(assign, a)
    assert np.allclose(cent, c, rtol=1e-6, atol=1e-7)


def test_pq_uneven_split_and_table_identity():
    s = KAT["pq_uneven_split"]
    w, _ = pxo.pq_layout(s["dim"], s["m"])
    assert list(w) == s["widths"]
    rng = np.random.default_rng(5)
    train = rng.standard_normal((512, 32)).astype(np.float32)
    books, _, _ = pxo.pq_train(train, 8)
    q = train[100]
    sq, dt = pxo.pq_tables(books, 32, 8, q)
    codes = pxo.pq_encode(books, 32, 8, train[:64])
    dec = pxo.pq_decode(books, 32, 8, codes)
    for code, rec in zip(codes, dec):
        via = pxo.pq_adc_squared(sq, 8, code)
        direct = pxo.squared_euclidean(q, rec)
        assert abs(via - direct) <= 1e-3 * max(direct, 1.0)


def test_sq_known_answers():
    c = KAT["sq_clamp"]
    mn, sc, inv = pxo.sq_train(np.array(c["training"], np.float32).reshape(-1, 1), pxo.RANGE_PER_DIMENSION)
    lo = pxo.sq_decode(mn, sc, 1, 1, 0, pxo.sq_encode(mn, inv, 1, 1, 0, [c["low"]]))
    hi = pxo.sq_decode(mn, sc, 1, 1, 0, pxo.sq_encode(mn, inv, 1, 1, 0, [c["high"]]))
    assert lo[0, 0] == c["low_decoded"] and hi[0, 0] == c["high_decoded"]
    k = KAT["sq_constant_dim"]
    mn, sc, inv = pxo.sq_train(np.array(k["training"], np.float32).reshape(-1, 2), pxo.RANGE_PER_DIMENSION)
    dec = pxo.sq_decode(mn, sc, 2, 1, 0, pxo.sq_encode(mn, inv, 2, 1, 0, k["probe"]))
    assert dec[0, 0] == k["decoded0"]
    # half-step bound and the U8/I8 lattices (scalar.rs:365-427)
    t = np.array([[i / 255.0, 1000.0 * i / 255.0] for i in range(256)], np.float32)
    mn, sc, inv = pxo.sq_train(t, pxo.RANGE_PER_DIMENSION)
    for ct in (pxo.CODE_U8, pxo.CODE_I8):
        dec = pxo.sq_decode(mn, sc, 2, 1, ct, pxo.sq_encode(mn, inv, 2, 1, ct, t))
        assert np.all(np.abs(dec[:, 0] - t[:, 0]) <= (1 / 255) / 2 + 1e-5)
        assert np.all(np.abs(dec[:, 1] - t[:, 1]) <= (1000 / 255) / 2 + 1e-5)
    u = pxo.sq_decode(mn, sc, 2, 1, 0, pxo.sq_encode(mn, inv, 2, 1, 0, t))
    i8 = pxo.sq_decode(mn, sc, 2, 1, 1, pxo.sq_encode(mn, inv, 2, 1, 1, t))
    assert np.array_equal(u, i8)


def _recall(exact, approx):
    return len(set(exact) & set(approx)) / len(exact)


def _topk(scores, k):
    order = sorted(range(len(scores)), key=lambda i: (np.float32(scores[i]).view(np.int32) ^ ((np.float32(scores[i]).view(np.int32) >> 31) & 0x7FFFFFFF), i))
    return order[:k]


def test_splitmix_fixture_recall_floors():
    """crates/proxima-quantize/tests/recall.rs:124-231 on the bit-identical splitmix fixture."""
    f = KAT["quantizer_recall_floors"]
    data = fixtures.splitmix_corpus(f["corpus"], f["corpus_seed"], f["dim"])
    queries = fixtures.splitmix_corpus(f["queries"], f["query_seed"], f["dim"])
    k = f["k"]
    ids, _, _ = pxo.flat_search(data, queries, k, pxo.EUCLIDEAN)
    truth = [list(map(int, r)) for r in ids]
    for mode, floor in ((pxo.RANGE_PER_DIMENSION, f["sq_per_dimension"]), (pxo.RANGE_GLOBAL, f["sq_global"])):
        mn, sc, inv = pxo.sq_train(data, mode)
        codes = pxo.sq_encode(mn, inv, f["dim"], mode, pxo.CODE_U8, data)
        rec = data_rec = pxo.sq_decode(mn, sc, f["dim"], mode, pxo.CODE_U8, codes)
        total = 0.0
        for qi, q in enumerate(queries):
            # asymmetric_squared_l2 == sequential L2 to the reconstruction
            s = [pxo.squared_euclidean_scalar(q, r) for r in data_rec]
            total += _recall(truth[qi], _topk(s, k))
        assert total / len(queries) >= floor, (mode, total / len(queries))


@pytest.mark.parametrize("m", [32, 16, 8])
def test_splitmix_fixture_pq_floors(m):
    f = KAT["quantizer_recall_floors"]
    data = fixtures.splitmix_corpus(f["corpus"], f["corpus_seed"], f["dim"])
    queries = fixtures.splitmix_corpus(f["queries"], f["query_seed"], f["dim"])
    k = f["k"]
    ids, _, _ = pxo.flat_search(data, queries, k, pxo.EUCLIDEAN)
    books, _, _ = pxo.pq_train(data, m, seed=f["pq_seed"])
    codes = pxo.pq_encode(books, f["dim"], m, data)
    total = 0.0
    for qi, q in enumerate(queries):
        sq, _ = pxo.pq_tables(books, f["dim"], m, q)
        s = sq.reshape(m, 256)[np.arange(m)[None, :], codes].astype(np.float32)
        # sequential f32 sum over subspaces (product.rs:580-588)
        acc = np.zeros(len(codes), np.float32)
        for j in range(m):
            acc = acc + s[:, j]
        total += _recall(list(map(int, ids[qi])), _topk(acc, k))
    assert total / len(queries) >= f["pq"][str(m)]


def test_ivfpq_train_and_search_properties():
    # crates/proxima-index/src/ivfpq.rs:1333-1349 and :1366-1404 (shape of the claims)
    data = fixtures.splitmix_corpus(2000, 11, 32)
    cent, books, list_of, codes, rep = pxo.ivfpq_train(data, 32, 16, seed=11)
    assert rep.sampled == 2000 and rep.populated_lists > 1
    assert np.bincount(list_of, minlength=len(cent)).sum() == 2000
    queries = data[::40]
    truth, _, _ = pxo.flat_search(data, queries, 10, pxo.EUCLIDEAN)
    prev = 0.0
    for nprobe in (1, 4, 16, 32):
        got, _, lens = pxo.ivfpq_search(None, cent, books, 16, list_of, codes, queries, 10, nprobe)
        r = np.mean([_recall(list(map(int, t)), list(map(int, g[:l]))) for t, g, l in zip(truth, got, lens)])
        assert r + 0.02 >= prev
        prev = r
    assert prev > 0.4
    base, _, lens = pxo.ivfpq_search(None, cent, books, 16, list_of, codes, queries, 10, 8)
    rr, _, lens2 = pxo.ivfpq_search(data, cent, books, 16, list_of, codes, queries, 10, 8, rerank=100)
    r0 = np.mean([_recall(list(map(int, t)), list(map(int, g))) for t, g in zip(truth, base)])
    r1 = np.mean([_recall(list(map(int, t)), list(map(int, g))) for t, g in zip(truth, rr)])
    assert r1 > r0
