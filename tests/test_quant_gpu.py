"""The proxima-quantize entry points on the GPU against the oracle, bit for bit:

* ProductQuantizer train / encode / decode / distance_table
  (crates/proxima-quantize/src/product.rs:198-439) through pxc_pq_*;
* ScalarQuantizer asymmetric_squared_l2 / asymmetric_inner_product
  (scalar.rs:298-327) through pxc_sq_asymmetric;
* kmeans drawing from the caller's ChaCha8Rng and advancing it in place
  (kmeans.rs:59-65), so that a second call continues the same stream;
* recall_at_k[_filtered] (crates/proxima-index/src/recall.rs:108-187): the
  per-query overlaps, the sequential f32 mean, the minimum and short results.
"""
import ctypes as C

import numpy as np
import pytest

from oracle import pxo
from proxima_b200 import fixtures
from proxima_b200.core import Metric, VectorSpace
from proxima_b200.errors import Configuration, NonFinite
from proxima_b200.index import FlatIndex, recall_at_k
from proxima_b200.ivfpq import IvfPqIndex
from proxima_b200.quantize import ChaCha8Rng, ProductQuantizer, kmeans
from proxima_b200.sq import CodeType, RangeMode, ScalarQuantizer

pytestmark = pytest.mark.gpu


def _bits_equal(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


@pytest.mark.parametrize("dim,m,n,iters", [(16, 4, 3000, 6), (64, 4, 5000, 5), (30, 7, 2000, 8), (8, 8, 200, 4)])
def test_pq_train_matches_oracle(dim, m, n, iters):
    """Widths 4 and 16 (the exact and tensor-core k-means paths), uneven widths
    (30 = 5+5+4+4+4+4+4), and fewer points than 256 codewords (padding)."""
    data = fixtures.sphere_blobs(n, dim, 30, 3 + dim, 4 + m, 0.1)
    pq = ProductQuantizer.train(dim, data, m, max_iterations=iters, seed=0x5EED + dim)
    books, inertia, its = pxo.pq_train(data, m, iters, seed=0x5EED + dim)
    assert _bits_equal(pq.codebooks, books)
    assert pq.training_inertia == inertia and pq.training_iterations == its


def test_pq_encode_decode_tables_match_oracle():
    dim, m = 40, 6  # widths 7,7,7,7,6,6
    rng = np.random.default_rng(3)
    books = rng.standard_normal(256 * dim).astype(np.float32)
    pq = ProductQuantizer(dim, m, books)
    vecs = rng.standard_normal((3000, dim)).astype(np.float32)
    vecs[5] = books[:dim]  # components taken from the codebook itself
    codes = pq.encode(vecs)
    assert np.array_equal(codes, pxo.pq_encode(books, dim, m, vecs))
    assert _bits_equal(pq.decode(codes), pxo.pq_decode(books, dim, m, codes))
    qs = rng.standard_normal((37, dim)).astype(np.float32)
    sq, dot = pq.distance_tables(qs)
    for i in range(len(qs)):
        rs, rd = pxo.pq_tables(books, dim, m, qs[i])
        assert _bits_equal(sq[i].reshape(-1), rs) and _bits_equal(dot[i].reshape(-1), rd)
    t = pq.distance_table(qs[0])
    rs, _ = pxo.pq_tables(books, dim, m, qs[0])
    for code in codes[:50]:
        assert np.float32(t.squared_l2(code)) == np.float32(pxo.pq_adc_squared(rs, m, code))


def test_pq_duplicate_codewords_tie_to_lower_index():
    """Padded codebooks repeat the last centroid; encode must pick the first copy."""
    dim, m = 8, 2
    data = fixtures.sphere_blobs(100, dim, 5, 1, 2, 0.1)  # 100 points < 256 codewords
    pq = ProductQuantizer.train(dim, data, m, max_iterations=5, seed=9)
    codes = pq.encode(data)
    assert codes.max() < 100
    assert np.array_equal(codes, pxo.pq_encode(pq.codebooks, dim, m, data))


def test_pq_argument_errors():
    data = np.ones((10, 8), np.float32)
    with pytest.raises(Configuration) as e:
        ProductQuantizer.train(8, data, 0)
    assert e.value.parameter == "subspaces"
    with pytest.raises(Configuration):
        ProductQuantizer.train(8, data, 9)
    with pytest.raises(Configuration) as e:
        ProductQuantizer.train(8, np.zeros((0, 8), np.float32), 2)
    assert e.value.parameter == "training"
    with pytest.raises(Configuration):
        ProductQuantizer.train(8, data, 2, max_iterations=0)
    bad = data.copy()
    bad[3, 5] = np.nan
    with pytest.raises(NonFinite) as e:
        ProductQuantizer.train(8, bad, 2)
    assert e.value.index == 5


@pytest.mark.parametrize("mode", [RangeMode.GLOBAL, RangeMode.PER_DIMENSION])
@pytest.mark.parametrize("code_type", [CodeType.U8, CodeType.I8])
def test_sq_asymmetric_matches_oracle(mode, code_type):
    dim = 70  # two shared-memory slabs, the second ragged
    data = fixtures.sphere_blobs(1500, dim, 20, 5, 6, 0.1)
    mn, sc, inv = pxo.sq_train(data, int(mode))
    quant = ScalarQuantizer(dim, mode, code_type, mn, sc, inv)
    codes = quant.encode(data[:700])
    qs = fixtures.sphere_blobs(19, dim, 20, 5, 16, 0.1)  # 19 queries: three blocks of 8, the last ragged
    l2 = quant.asymmetric(qs, codes, Metric.EUCLIDEAN)
    ip = quant.asymmetric(qs, codes, Metric.INNER_PRODUCT)
    assert _bits_equal(ip, quant.asymmetric(qs, codes, Metric.COSINE))
    L = pxo.lib()
    for i in range(len(qs)):
        q = np.ascontiguousarray(qs[i])
        for j in range(0, len(codes), 7):
            c = np.ascontiguousarray(codes[j])
            want_l2 = L.pxo_sq_asymmetric_squared_l2(mn.ctypes.data, sc.ctypes.data, dim, int(mode),
                                                     int(code_type), q.ctypes.data, c.ctypes.data)
            want_ip = L.pxo_sq_asymmetric_inner_product(mn.ctypes.data, sc.ctypes.data, dim, int(mode),
                                                        int(code_type), q.ctypes.data, c.ctypes.data)
            assert np.float32(l2[i, j]).view(np.uint32) == np.float32(want_l2).view(np.uint32)
            assert np.float32(ip[i, j]).view(np.uint32) == np.float32(want_ip).view(np.uint32)


def _oracle_rng_word_pos(r) -> int:
    block = (r.counter - 4 + r.index // 16) & ((1 << 64) - 1)
    return block * 16 + r.index % 16


def test_kmeans_draws_from_and_advances_the_callers_rng():
    """Two k-means++ runs from one generator equal the oracle's two runs from one
    pxo_rng; the generator's word position after each equals the oracle's."""
    dim = 12
    a = fixtures.sphere_blobs(3000, dim, 25, 8, 9, 0.1)
    b = fixtures.sphere_blobs(2000, dim, 25, 8, 10, 0.1)
    rng = ChaCha8Rng.seed_from_u64(0xC0FFEE)
    r = pxo.Rng()
    L = pxo.lib()
    L.pxo_rng_seed_from_u64(C.byref(r), 0xC0FFEE)
    for pts, k in ((a, 40), (b, 33)):
        got = kmeans(pts, dim, k, 6, rng=rng, want_assignment=True)
        cent = np.zeros((k, dim), np.float32)
        assign = np.zeros(len(pts), np.uint32)
        inertia, iters = C.c_double(), C.c_uint64()
        L.pxo_kmeans(pts.ctypes.data, len(pts), dim, k, 6, None, 0, C.byref(r), cent.ctypes.data,
                     assign.ctypes.data, C.byref(inertia), C.byref(iters), pxo.threads())
        assert _bits_equal(got.centroids, cent) and np.array_equal(got.assignment, assign)
        assert got.inertia == inertia.value and got.iterations == iters.value
        assert rng.get_word_pos() == _oracle_rng_word_pos(r) > 0
    # an injected init draws nothing
    pos = rng.get_word_pos()
    kmeans(a, dim, 10, 3, rng=rng, init=a[:10])
    assert rng.get_word_pos() == pos


def test_kmeans_without_init_needs_a_generator():
    from proxima_b200 import _native as N
    from proxima_b200.index import Context

    pts = np.ones((10, 4), np.float32)
    cent = np.zeros((4, 4), np.float32)
    with pytest.raises(Configuration):
        N.call("pxc_kmeans", Context.default().handle, N.ptr(pts), 10, 4, 4, 3, None, None, N.ptr(cent), None,
               None)


class _IvfCandidate:
    """An approximate index for recall_at_k: IVF-PQ with a small nprobe."""

    def __init__(self, ivf: IvfPqIndex, nprobe: int):
        self.ivf, self.nprobe = ivf, nprobe

    def search_batch(self, queries, k, filter=None):
        from proxima_b200.core import SearchResult

        ids, dist, lens = self.ivf.search_batch(queries, k, self.nprobe, rerank=0)
        return [[SearchResult(int(ids[q, j]), float(dist[q, j])) for j in range(lens[q])] for q in range(len(lens))]


def test_recall_at_k_matches_oracle():
    dim, n, nlist, m, k = 32, 6000, 32, 8, 10
    data = fixtures.sphere_blobs(n, dim, 40, 21, 22, 0.1)
    queries = fixtures.sphere_blobs(150, dim, 40, 21, 23, 0.1)
    cent, books, list_of, codes, _ = pxo.ivfpq_train(data, nlist, m, 5, 3000, 0x77)
    ivf = IvfPqIndex(dim, nlist, m, Metric.EUCLIDEAN)
    ivf.from_parts(cent, books)
    ivf.set_store(data)
    ivf.set_codes(list_of, codes)
    truth = FlatIndex.from_array(VectorSpace(dim, Metric.EUCLIDEAN), data)
    rep = recall_at_k(_IvfCandidate(ivf, 2), truth, queries, k)
    eids, _, elen = pxo.flat_search(data, queries, k, pxo.EUCLIDEAN)
    aids, _, alen = pxo.ivfpq_search(data, cent, books, m, list_of, codes, queries, k, 2, 0, pxo.EUCLIDEAN)
    per = []
    short = 0
    for q in range(len(queries)):
        e = eids[q, :elen[q]]
        a = aids[q, :alen[q]]
        short += int(len(a) < len(e))
        per.append(np.float32(np.float32(sum(1 for x in a if x in set(e.tolist()))) / np.float32(len(e))))
    total = np.float32(0.0)
    for r in per:
        total = np.float32(total + r)
    assert rep.queries == len(queries) and rep.short_results == short
    assert np.array_equal(np.asarray(rep.per_query, np.float32), np.asarray(per, np.float32))
    assert np.float32(rep.mean) == np.float32(total / np.float32(len(per)))
    assert np.float32(rep.min) == min(per)
    assert 0.2 < rep.mean < 1.0
    with pytest.raises(Configuration):
        recall_at_k(_IvfCandidate(ivf, 2), truth, np.zeros(dim + 1, np.float32), k)
    empty = recall_at_k(_IvfCandidate(ivf, 2), truth, np.zeros(0, np.float32), k)
    assert empty.queries == 0 and empty.mean == 0.0 and empty.min == 0.0
    ivf.close()
    truth.close()
