"""The allocation-free flat search (pxc_flat_search_noalloc) against the regular entry point.

Some callers cannot allocate device memory while they search — a runtime that
has reserved the whole GPU for its own pool, or a serving loop that cannot pay
for the device-wide synchronisation of cudaMalloc/cudaFree. For them the
library offers one entry point whose scratch lives in a fixed device array.
This file is collected last on purpose, so a failure here comes after every
other test has run. It must pass alone and after the others: the array keeps
the previous call's contents, and each call must reset what it relies on.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _search(fn, handle, q, k, torch):
    nq = q.shape[0]
    ids = torch.full((nq, k), -1, dtype=torch.int64, device="cuda")
    dist = torch.full((nq, k), float("nan"), dtype=torch.float32, device="cuda")
    lens = torch.full((nq,), -1, dtype=torch.int32, device="cuda")
    from proxima_b200 import _native as N
    N.call(fn, handle, q.data_ptr(), nq, k, *( [None] if fn == "pxc_flat_search_device" else [] ),
           ids.data_ptr(), dist.data_ptr(), lens.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return ids.cpu().numpy(), dist.cpu().numpy(), lens.cpu().numpy()


def test_noalloc_search_matches_the_regular_entry_point_on_two_calls():
    import torch
    from proxima_b200 import _native as N
    from proxima_b200 import fixtures
    from proxima_b200.index import Context

    db = fixtures.blobs_u8(40_000, 128, 512, fixtures.C2_CENTRES, fixtures.C2_BASE)
    ctx = Context.default()
    h = N.vp()
    N.call("pxc_flat_create", ctx.handle, 128, 0, C.byref(h))
    try:
        N.call("pxc_flat_sync", h, N.ptr(db), None, None, 0, len(db))
        assert N.load().pxc_flat_len(h) == len(db)  # builds the mirror (this allocates)
        for call, (nq, k, seed) in enumerate([(600, 10, fixtures.C2_QUERIES), (333, 16, fixtures.C2_QUERIES + 7)]):
            q = torch.from_numpy(fixtures.blobs_u8(nq, 128, 512, fixtures.C2_CENTRES, seed)).cuda()
            ref = _search("pxc_flat_search_device", h, q, k, torch)
            got = _search("pxc_flat_search_noalloc", h, q, k, torch)
            assert np.array_equal(got[2], ref[2]), f"call {call}: lengths"
            for i in range(nq):
                n = int(ref[2][i])
                assert np.array_equal(got[0][i, :n], ref[0][i, :n]), f"call {call} query {i}: ids"
                assert np.array_equal(got[1][i, :n].view(np.uint32), ref[1][i, :n].view(np.uint32)), f"call {call} query {i}"
        # limits are rejected with a clear error, before any work
        from proxima_b200.errors import Capacity, Configuration
        big = torch.zeros((2049, 128), dtype=torch.float32, device="cuda")
        with pytest.raises(Capacity):
            _search("pxc_flat_search_noalloc", h, big, 10, torch)
        with pytest.raises(Configuration):
            _search("pxc_flat_search_noalloc", h, big[:4], 17, torch)
    finally:
        N.load().pxc_flat_destroy(h)


@pytest.mark.parametrize("k", [1, 4])
def test_noalloc_search_at_its_limits_matches_the_oracle(k):
    """At the entry point's limits — 2,048 queries, dim 256 (two K blocks), a
    120k-row store, so the split count is clamped to the array's 32 — the ids
    and distance bits equal the oracle's exact search and the regular entry
    point's, on two calls in a row."""
    import torch
    from oracle import pxo
    from proxima_b200 import _native as N
    from proxima_b200 import fixtures
    from proxima_b200.index import Context

    dim, n, nq = 256, 120_000, 2048
    db = fixtures.blobs_u8(n, dim, 512, fixtures.C2_CENTRES + 3, fixtures.C2_BASE + 3)
    ctx = Context.default()
    h = N.vp()
    N.call("pxc_flat_create", ctx.handle, dim, 0, C.byref(h))
    try:
        N.call("pxc_flat_sync", h, N.ptr(db), None, None, 0, n)
        assert N.load().pxc_flat_len(h) == n
        for call in range(2):
            qh = fixtures.blobs_u8(nq, dim, 512, fixtures.C2_CENTRES + 3, fixtures.C2_QUERIES + 11 + call)
            q = torch.from_numpy(qh).cuda()
            got = _search("pxc_flat_search_noalloc", h, q, k, torch)
            ref = _search("pxc_flat_search_device", h, q, k, torch)
            ri, rd, rl = pxo.flat_search(db, qh, k, pxo.EUCLIDEAN)
            assert np.array_equal(got[2], rl) and np.array_equal(ref[2], rl), f"call {call}: lengths"
            assert np.array_equal(got[0], ri.astype(np.int64)), f"call {call}: ids"
            assert np.array_equal(got[1].view(np.uint32), rd.view(np.uint32)), f"call {call}: distances"
            assert np.array_equal(got[0], ref[0]) and np.array_equal(got[1].view(np.uint32), ref[1].view(np.uint32))
    finally:
        N.load().pxc_flat_destroy(h)
