"""Host mirror of proxima-index's IvfPqIndex on the B200 backend (pxc_ivfpq).

Holds the parts the reference's IvfPqIndex holds (crates/proxima-index/src/ivfpq.rs):
coarse centroids and product-quantizer codebooks (``from_parts``), the slot
store (prepared vectors, VectorIds, live flags) and the per-slot list
assignment and codes. ``search_batch`` is ``search_with_nprobe`` for a batch
of prepared queries, run on the GPU, with the filter given as a slot bitmap.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _native as N
from .core import Metric


class IvfPqIndex:
    def __init__(self, dim: int, nlist: int, subspaces: int, metric: Metric = Metric.EUCLIDEAN, context=None):
        from .index import Context

        self.ctx = context or Context.default()
        self.dim, self.nlist, self.m = dim, nlist, subspaces
        self.metric = Metric(metric)
        h = N.vp()
        N.call("pxc_ivfpq_create", self.ctx.handle, dim, int(self.metric), nlist, subspaces, C.byref(h))
        self.handle = h
        self.nslots = 0

    def close(self) -> None:
        if getattr(self, "handle", None):
            N.load().pxc_ivfpq_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def from_parts(self, centroids, codebooks) -> "IvfPqIndex":
        cent = np.ascontiguousarray(centroids, dtype=np.float32)
        books = np.ascontiguousarray(codebooks, dtype=np.float32)
        if cent.size != self.nlist * self.dim or books.size != 256 * self.dim:
            raise ValueError("parts do not match (nlist, dim)")
        N.call("pxc_ivfpq_set_parts", self.handle, N.ptr(cent), N.ptr(books))
        return self

    def set_store(self, vectors=None, ids=None, live=None, nslots: int | None = None) -> None:
        v = None if vectors is None else np.ascontiguousarray(vectors, dtype=np.float32)
        n = nslots if nslots is not None else (len(v) if v is not None else len(ids))
        i = None if ids is None else np.ascontiguousarray(ids, dtype=np.uint64)
        lv = None if live is None else np.ascontiguousarray(live, dtype=np.uint8)
        N.call("pxc_ivfpq_set_store", self.handle, N.ptr(v), N.ptr(i), N.ptr(lv), n)
        self.nslots = n

    def set_codes(self, list_of, codes) -> None:
        lo = np.ascontiguousarray(list_of, dtype=np.uint32)
        cd = np.ascontiguousarray(codes, dtype=np.uint8)
        N.call("pxc_ivfpq_set_codes", self.handle, N.ptr(lo), N.ptr(cd))

    def search_batch(self, queries, k: int, nprobe: int, rerank: int = 0, bitmap=None):
        q = np.ascontiguousarray(queries, dtype=np.float32).reshape(-1, self.dim)
        nq = len(q)
        kk = max(k, 1)
        ids = np.zeros((nq, kk), dtype=np.uint64)
        dist = np.zeros((nq, kk), dtype=np.float32)
        lens = np.zeros(nq, dtype=np.uint32)
        bm = None if bitmap is None else np.ascontiguousarray(bitmap, dtype=np.uint64)
        N.call("pxc_ivfpq_search", self.handle, N.ptr(q), nq, k, nprobe, rerank, N.ptr(bm), N.ptr(ids),
               N.ptr(dist), N.ptr(lens))
        return ids[:, :k], dist[:, :k], lens
