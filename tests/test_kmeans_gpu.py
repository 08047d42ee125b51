"""k-means on the GPU (pxc_kmeans) against the oracle's restatement of
crates/proxima-quantize/src/kmeans.rs, bit for bit: centroids, assignments,
inertia and iteration count, on both assignment paths (exact CUDA-core and
tensor-core screening + exact re-scoring), with k-means++ and injected seeds,
empty-cluster re-seeding, duplicate centroids (ties, screening overflow),
the k clamp and the degenerate shapes the reference handles.
"""

import numpy as np
import pytest

from oracle import pxo
from proxima_b200 import fixtures
from proxima_b200.index import Context
from proxima_b200.quantize import kmeans

pytestmark = pytest.mark.gpu


def _same(got, cent, assign, inertia, iters, label=""):
    assert got.iterations == iters, f"{label}: iterations {got.iterations} != {iters}"
    assert got.centroids.shape == cent.shape, label
    bad = np.flatnonzero(got.centroids.view(np.uint32) != cent.view(np.uint32))
    assert bad.size == 0, f"{label}: {bad.size} centroid values differ, first at {bad[:5]}"
    if got.assignment is not None:
        diff = np.flatnonzero(got.assignment != assign)
        assert diff.size == 0, f"{label}: {diff.size} assignments differ, first at {diff[:5]}"
    assert got.inertia == inertia, f"{label}: inertia {got.inertia!r} != {inertia!r}"


def _blobs(n, dim, nblobs, seed, sigma=0.05):
    return fixtures.sphere_blobs(n, dim, nblobs, fixtures.C3_CENTRES + seed, fixtures.C3_POINTS + seed, sigma)


def test_small_exact_path_with_kmeanspp_matches_oracle():
    pts = _blobs(3000, 8, 24, 1, sigma=0.2)
    for seed in (0, 7, 0x00C0FFEE):
        cent, assign, inertia, iters = pxo.kmeans(pts, 32, 25, seed=seed)
        got = kmeans(pts, 8, 32, 25, seed=seed, want_assignment=True)
        assert got.path == 0
        _same(got, cent, assign, inertia, iters, f"seed {seed}")


def test_injected_init_exact_path():
    pts = _blobs(5000, 40, 64, 2, sigma=0.1)
    init = fixtures.c3_init(pts, 100, seed=5)
    cent, assign, inertia, iters = pxo.kmeans(pts, 100, 12, init=init)
    got = kmeans(pts, 40, 100, 12, init=init, want_assignment=True)
    assert got.path == 0
    _same(got, cent, assign, inertia, iters)


@pytest.mark.parametrize("dim", [96, 64, 128, 17])
def test_tensor_path_matches_oracle(dim):
    # C3-shaped data: more centroids than blobs, so many blobs are split and
    # their points sit near Voronoi boundaries (the screening's hard case).
    pts = _blobs(16384, dim, 400, 3, sigma=0.05)
    init = fixtures.c3_init(pts, 512, seed=11)
    cent, assign, inertia, iters = pxo.kmeans(pts, 512, 6, init=init)
    got = kmeans(pts, dim, 512, 6, init=init, want_assignment=True)
    assert got.path == 1
    _same(got, cent, assign, inertia, iters, f"dim {dim}")


def test_tensor_path_equals_forced_exact_path():
    pts = _blobs(8192, 96, 300, 4)
    init = fixtures.c3_init(pts, 300, seed=3)
    a = kmeans(pts, 96, 300, 5, init=init, want_assignment=True)
    ctx = Context.default()
    ctx.set_option("kmeans_exact", 1)
    try:
        b = kmeans(pts, 96, 300, 5, init=init, want_assignment=True)
    finally:
        ctx.set_option("kmeans_exact", 0)
    assert a.path == 1 and b.path == 0
    assert np.array_equal(a.centroids.view(np.uint32), b.centroids.view(np.uint32))
    assert np.array_equal(a.assignment, b.assignment)
    assert a.inertia == b.inertia and a.iterations == b.iterations


def test_duplicate_centroids_tie_to_lower_index_and_rescan():
    pts = _blobs(6000, 32, 40, 5, sigma=0.08)
    init = fixtures.c3_init(pts, 300, seed=9).copy()
    init[10:30] = init[10]  # 20 identical centroids: ties, and more candidates than the screen keeps
    init[200:203] = init[150]
    cent, assign, inertia, iters = pxo.kmeans(pts, 300, 4, init=init)
    got = kmeans(pts, 32, 300, 4, init=init, want_assignment=True)
    assert got.path == 1
    assert got.rescanned > 0
    _same(got, cent, assign, inertia, iters)


@pytest.mark.parametrize("k", [40, 260])
def test_empty_clusters_are_reseeded_like_the_reference(k):
    pts = _blobs(4000, 24, 30, 6, sigma=0.1)
    init = fixtures.c3_init(pts, k, seed=4).copy()
    init[3] = 50.0   # far from every point: empty after the first assignment
    init[k - 2] = -40.0
    cent, assign, inertia, iters = pxo.kmeans(pts, k, 8, init=init)
    got = kmeans(pts, 24, k, 8, init=init, want_assignment=True)
    assert got.reseeded >= 2
    assert got.path == (1 if k >= 256 else 0)
    _same(got, cent, assign, inertia, iters, f"k {k}")


def test_integer_data_c2_shape():
    pts = fixtures.blobs_u8(6000, 128, 64, fixtures.C2_CENTRES, fixtures.C2_BASE)
    init = fixtures.c3_init(pts, 256, seed=2)
    cent, assign, inertia, iters = pxo.kmeans(pts, 256, 5, init=init)
    got = kmeans(pts, 128, 256, 5, init=init, want_assignment=True)
    assert got.path == 1
    _same(got, cent, assign, inertia, iters)


def test_kmeanspp_on_the_tensor_path():
    pts = _blobs(6000, 48, 200, 7, sigma=0.05)
    cent, assign, inertia, iters = pxo.kmeans(pts, 300, 4, seed=0x5EED)
    got = kmeans(pts, 48, 300, 4, seed=0x5EED, want_assignment=True)
    assert got.path == 1
    _same(got, cent, assign, inertia, iters)


def test_convergence_stops_early_and_counts_the_last_pass():
    pts = _blobs(2000, 16, 5, 8, sigma=0.02)
    cent, assign, inertia, iters = pxo.kmeans(pts, 5, 50, seed=1)
    got = kmeans(pts, 16, 5, 50, seed=1, want_assignment=True)
    assert iters < 50
    _same(got, cent, assign, inertia, iters)


def test_clamp_degenerate_and_errors():
    from proxima_b200.errors import NonFinite

    pts = _blobs(10, 6, 3, 9, sigma=0.3)
    cent, assign, inertia, iters = pxo.kmeans(pts, 50, 10, seed=3)
    got = kmeans(pts, 6, 50, 10, seed=3, want_assignment=True)
    assert got.centroids.shape == (10, 6)
    _same(got, cent, assign, inertia, iters)
    # identical points: total is 0 every round, uniform picks
    same = np.ones((64, 5), np.float32)
    cent, assign, inertia, iters = pxo.kmeans(same, 4, 10, seed=2)
    got = kmeans(same, 5, 4, 10, seed=2, want_assignment=True)
    _same(got, cent, assign, inertia, iters)
    # no points / zero dim / no iterations
    got = kmeans(np.zeros(0, np.float32), 4, 3, 10)
    assert got.centroids.shape == (1, 4) and not got.centroids.any() and got.iterations == 0
    got = kmeans(pts, 6, 3, 0, seed=3, want_assignment=True)
    cent, assign, inertia, iters = pxo.kmeans(pts, 3, 0, seed=3)
    _same(got, cent, assign, inertia, iters)
    bad = pts.copy()
    bad[4, 2] = np.nan
    with pytest.raises(NonFinite):
        kmeans(bad, 6, 3, 5)


def test_device_entry_point_matches_host_entry_point():
    import torch

    pts = _blobs(8000, 96, 300, 10)
    init = fixtures.c3_init(pts, 256, seed=1)
    a = kmeans(pts, 96, 256, 4, init=init, want_assignment=True)
    b = kmeans(torch.from_numpy(pts).cuda(), 96, 256, 4, init=init, want_assignment=True)
    torch.cuda.synchronize()
    assert np.array_equal(a.centroids.view(np.uint32), b.centroids.view(np.uint32))
    assert np.array_equal(a.assignment, b.assignment)
    assert a.inertia == b.inertia and a.iterations == b.iterations


def test_c3_at_the_configuration_size():
    """C3 exactly as bench.py trains it (1M x 96 unit-sphere blobs, k = 4096, the
    seeded-sample start), cut to its first two Lloyd iterations so the oracle
    finishes in about a minute on the host's cores: centroids, assignments and
    inertia bit-identical to the oracle's."""
    pts = fixtures.c3_points(1_000_000, 96)
    init = fixtures.c3_init(pts, 4096)
    cent, assign, inertia, iters = pxo.kmeans(pts, 4096, 2, init=init)
    got = kmeans(pts, 96, 4096, 2, init=init, want_assignment=True)
    assert got.path == 1  # the tensor-core screen with exact re-scoring
    _same(got, cent, assign, inertia, iters, "C3 full size, 2 iterations")
