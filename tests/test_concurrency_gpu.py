"""Concurrent searches, as the reference's store issues them: `search` runs
under the collection's read lock (crates/proxima-store/src/collection.rs:373-383),
so several threads may search one index, or several indexes of one context, at
once. Every result must equal the serial one, and each call must see only the
failures of its own kernels.

* two flat handles on one context searched from two host threads on the
  tensor-core scan (each handle owns its device error word);
* one flat handle (fp32 scan, k = 30, which returns before its kernels finish) and one
  IVF-PQ handle searched on two CUDA streams with interleaved calls: each
  handle passes its scratch from one search to the next in stream order.
"""
import threading

import numpy as np
import pytest

from oracle import pxo
from proxima_b200 import _native as N
from proxima_b200 import fixtures
from proxima_b200.core import Metric, VectorSpace
from proxima_b200.index import Context, FlatIndex
from proxima_b200.ivfpq import IvfPqIndex

pytestmark = pytest.mark.gpu


def _same(a, b, label):
    assert np.array_equal(a[2], b[2]), f"{label}: lengths"
    assert np.array_equal(a[0], b[0]), f"{label}: ids"
    assert np.array_equal(np.asarray(a[1]).view(np.uint32), np.asarray(b[1]).view(np.uint32)), f"{label}: distances"


def test_two_flat_handles_on_one_context_from_two_threads():
    ctx = Context(0)
    dbs = [fixtures.blobs_u8(60_000, 128, 256, fixtures.C2_CENTRES + i, fixtures.C2_BASE + i) for i in (1, 2)]
    idxs = [FlatIndex.from_array(VectorSpace(128, Metric.EUCLIDEAN), db, ctx=ctx) for db in dbs]
    qs = [fixtures.blobs_u8(700, 128, 256, fixtures.C2_CENTRES + i, fixtures.C2_QUERIES + i) for i in (1, 2)]
    serial = [idx.search_prepared_batch(q, 10) for idx, q in zip(idxs, qs)]
    assert all(idx.device_path() == 1 for idx in idxs)
    errors, results = [], [[], []]

    def worker(t):
        try:
            for _ in range(12):
                results[t].append(idxs[t].search_prepared_batch(qs[t], 10))
        except Exception as e:  # surfaced below
            errors.append(e)

    threads = [threading.Thread(target=worker, args=(t,)) for t in (0, 1)]
    for th in threads:
        th.start()
    for th in threads:
        th.join()
    assert not errors, errors
    for t in (0, 1):
        for r in results[t]:
            _same(r, serial[t], f"handle {t}")
    ri, rd, rl = pxo.flat_search(dbs[0], qs[0], 10, pxo.EUCLIDEAN)
    _same(serial[0], (ri, rd, rl), "vs oracle")
    for idx in idxs:
        idx.close()
    ctx.close()


def _flat_device(idx, dq, k, stream, torch):
    nq = dq.shape[0]
    ids = torch.empty((nq, k), dtype=torch.int64, device="cuda")
    dist = torch.empty((nq, k), dtype=torch.float32, device="cuda")
    lens = torch.empty((nq,), dtype=torch.int32, device="cuda")
    N.call("pxc_flat_search_device", idx.handle, dq.data_ptr(), nq, k, None, ids.data_ptr(), dist.data_ptr(),
           lens.data_ptr(), stream.cuda_stream)
    return ids, dist, lens


def _ivf_device(ivf, dq, k, nprobe, rerank, stream, torch):
    nq = dq.shape[0]
    ids = torch.empty((nq, k), dtype=torch.int64, device="cuda")
    dist = torch.empty((nq, k), dtype=torch.float32, device="cuda")
    lens = torch.empty((nq,), dtype=torch.int32, device="cuda")
    ivf.search_device(dq, k, nprobe, rerank, ids, dist, lens, stream.cuda_stream)
    return ids, dist, lens


def _host(t):
    ids, dist, lens = t
    return ids.cpu().numpy().view(np.uint64), dist.cpu().numpy(), lens.cpu().numpy().view(np.uint32)


def test_interleaved_searches_on_two_streams_equal_serial():
    import torch

    dim, n = 64, 40_000
    data = fixtures.sphere_blobs(n, dim, 64, 31, 32, 0.1)  # not integers: the fp32 flat scan
    batches = [fixtures.sphere_blobs(300 + 37 * i, dim, 64, 31, 40 + i, 0.1) for i in range(6)]
    flat = FlatIndex.from_array(VectorSpace(dim, Metric.EUCLIDEAN), data)
    kf = 30  # beyond the f16 screen's k: the fp32 scan, which returns before its kernels finish
    cent, books, list_of, codes, _ = pxo.ivfpq_train(data, 64, 8, 4, 8000, 0x31)
    ivf = IvfPqIndex(dim, 64, 8, Metric.EUCLIDEAN)
    ivf.from_parts(cent, books)
    ivf.set_store(data)
    ivf.set_codes(list_of, codes)
    serial_flat = [flat.search_prepared_batch(b, kf) for b in batches]
    serial_ivf = [ivf.search_batch(b, 10, 8, 200) for b in batches]
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    dqs = [torch.from_numpy(b).cuda() for b in batches]
    torch.cuda.synchronize()
    out_flat, out_ivf = [], []
    for i, dq in enumerate(dqs):  # consecutive searches alternate between the two streams
        s = streams[i % 2]
        out_flat.append(_flat_device(flat, dq, kf, s, torch))
        out_ivf.append(_ivf_device(ivf, dq, 10, 8, 200, streams[(i + 1) % 2], torch))
    torch.cuda.synchronize()
    for i in range(len(batches)):
        _same(_host(out_flat[i]), serial_flat[i], f"flat batch {i}")
        _same(_host(out_ivf[i]), serial_ivf[i], f"ivf batch {i}")
    flat.close()
    ivf.close()
