"""CPU checks of the SQ composition's host-side pieces: the oracle's restatement
of the int8 over-fetch + exact re-rank against the exact filtered FlatIndex
answer (crates/proxima-index/src/flat.rs:153-169), its query quantization, and
the rank-order fold of per-shard quantizer ranges (combine_ranges) against one
pass of ScalarQuantizer::train (crates/proxima-quantize/src/scalar.rs:141-195)."""
import numpy as np

from oracle import pxo
from proxima_b200 import fixtures
from proxima_b200.sq import combine_ranges


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def test_sharded_ranges_fold_equals_one_pass():
    rng = np.random.default_rng(11)
    t = rng.standard_normal((3000, 9)).astype(np.float32)
    t[:, 0] = np.abs(t[:, 0])
    t[1200, 0] = -0.0  # the first zero of column 0 lies in the second shard
    t[2500, 0] = 0.0
    t[:, 1] = np.abs(t[:, 1])
    t[100, 1] = 0.0  # column 1: +0 first, -0 later
    t[2900, 1] = -0.0
    mn, sc, inv = pxo.sq_train(t, pxo.RANGE_PER_DIMENSION)
    lows, highs = [], []
    for a, b in ((0, 1000), (1000, 2000), (2000, 3000)):
        m, s, _ = pxo.sq_train(t[a:b], pxo.RANGE_PER_DIMENSION)
        lows.append(m)
        highs.append(m + s * np.float32(255.0))  # only min is compared bit for bit below
    cmn, _, _ = combine_ranges(lows, highs)
    assert np.array_equal(_bits(cmn), _bits(mn))


def test_query_s8_uses_the_full_range():
    sc = np.full(16, 0.01, np.float32)
    q = np.linspace(-1, 1, 16).astype(np.float32)
    q8 = pxo.sq_query_s8(sc, 16, pxo.RANGE_PER_DIMENSION, q)
    assert q8.max() == 127 and q8.min() == -127
    assert np.all(pxo.sq_query_s8(sc, 16, pxo.RANGE_PER_DIMENSION, np.zeros(16, np.float32)) == 0)


def test_sq_search_equals_exact_filtered_flat_on_separated_data():
    dim, n = 48, 6000
    data = fixtures.sphere_blobs(n, dim, 60, 31, 32, 0.03)
    years = fixtures.uniform_int(n, 33, 2000, 30)
    queries = fixtures.sphere_blobs(40, dim, 60, 31, 34, 0.03)
    mn, sc, inv = pxo.sq_train(data, pxo.RANGE_PER_DIMENSION)
    codes = pxo.sq_encode(mn, inv, dim, pxo.RANGE_PER_DIMENSION, pxo.CODE_I8, data)
    acc = years >= 2015
    gi, gd, gl = pxo.sq_search(sc, pxo.RANGE_PER_DIMENSION, codes, data, queries, 10, 100, pxo.COSINE,
                               accepted=acc.astype(np.uint8))
    words = np.zeros((n + 63) // 64, np.uint64)
    for s in np.nonzero(acc)[0]:
        words[s >> 6] |= np.uint64(1) << np.uint64(s & 63)
    ri, rd, rl = pxo.flat_search(data, queries, 10, pxo.COSINE, bitmap=words)
    assert np.array_equal(gl, rl) and np.array_equal(gi, ri) and np.array_equal(_bits(gd), _bits(rd))
