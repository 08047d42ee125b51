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

    @classmethod
    def adopt(cls, handle, context, dim: int, nlist: int, subspaces: int, metric: Metric, nslots: int) -> "IvfPqIndex":
        """An index around an existing pxc_ivfpq handle (a snapshot load's); it owns the handle."""
        self = cls.__new__(cls)
        self.ctx = context
        self.dim, self.nlist, self.m = dim, nlist, subspaces
        self.metric = Metric(metric)
        self.handle = handle
        self.nslots = nslots
        return self

    def close(self) -> None:
        if getattr(self, "_columns", None) is not None:
            self._columns.close()
            self._columns = None
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

    def set_store_device(self, vectors, ids=None, live=None) -> None:
        """The store with the vectors already on the GPU (a CUDA torch tensor, n x dim)."""
        n = vectors.shape[0]
        i = None if ids is None else np.ascontiguousarray(ids, dtype=np.uint64)
        lv = None if live is None else np.ascontiguousarray(live, dtype=np.uint8)
        N.call("pxc_ivfpq_set_store_device", self.handle, vectors.contiguous().data_ptr(), N.ptr(i), N.ptr(lv), n)
        self.nslots = n

    def set_codes(self, list_of, codes) -> None:
        lo = np.ascontiguousarray(list_of, dtype=np.uint32)
        cd = np.ascontiguousarray(codes, dtype=np.uint8)
        N.call("pxc_ivfpq_set_codes", self.handle, N.ptr(lo), N.ptr(cd))

    def encode_all(self) -> None:
        N.call("pxc_ivfpq_encode_all", self.handle)

    def train(self, training_sample: int = 100_000, max_iterations: int = 25, seed: int = 0x1FF9C0D):
        """IvfPqIndex::train on the GPU; returns the TrainingReport fields as a dict."""
        rep = N.PxcIvfpqReport()
        N.call("pxc_ivfpq_train", self.handle, training_sample, max_iterations, seed, C.byref(rep))
        self.nlist = int(rep.produced)
        self.report = {f: getattr(rep, f) for f, _ in N.PxcIvfpqReport._fields_}
        return dict(self.report)

    def parts(self):
        """(centroids, codebooks, list_of, codes) as the index holds them."""
        cent = np.zeros((self.nlist, self.dim), dtype=np.float32)
        books = np.zeros(256 * self.dim, dtype=np.float32)
        list_of = np.zeros(max(self.nslots, 1), dtype=np.uint32)
        codes = np.zeros((max(self.nslots, 1), self.m), dtype=np.uint8)
        nl = C.c_uint32()
        N.call("pxc_ivfpq_get_parts", self.handle, N.ptr(cent), N.ptr(books), N.ptr(list_of), N.ptr(codes), C.byref(nl))
        return cent, books, list_of[:self.nslots], codes[:self.nslots]

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

    def set_metadata(self, metadata) -> None:
        """Per-slot metadata dicts (None or {} for none), for MetadataFilter searches."""
        self._metadata = list(metadata)
        self._col_fields = set()

    def search_where(self, queries, k: int, nprobe: int, rerank: int, flt):
        """search_with_nprobe with a MetadataFilter evaluated on the device (pxc_ivfpq_search_where)."""
        from .filters import DeviceColumns

        meta = getattr(self, "_metadata", [])
        if getattr(self, "_columns", None) is None:
            self._columns = DeviceColumns(self.ctx)
            self._col_fields = set()
        for field in flt.fields():
            if field not in self._col_fields:
                self._columns.set_values(field, [(m or {}).get(field) for m in meta], 0)
                self._col_fields.add(field)
        conds, nc, ops, no = flt.compile(self._columns)
        q = np.ascontiguousarray(queries, dtype=np.float32).reshape(-1, self.dim)
        nq = len(q)
        ids = np.zeros((nq, max(k, 1)), dtype=np.uint64)
        dist = np.zeros((nq, max(k, 1)), dtype=np.float32)
        lens = np.zeros(nq, dtype=np.uint32)
        N.call("pxc_ivfpq_search_where", self.handle, self._columns.handle, conds, nc, ops, no, N.ptr(q), nq, k,
               nprobe, rerank, N.ptr(ids), N.ptr(dist), N.ptr(lens))
        return ids[:, :k], dist[:, :k], lens

    def search_device(self, d_queries, k: int, nprobe: int, rerank: int, d_ids, d_dist, d_lens, stream: int,
                      d_bitmap=None) -> None:
        """Device-buffer search (torch tensors), enqueued on `stream`."""
        N.call("pxc_ivfpq_search_device", self.handle, d_queries.data_ptr(), d_queries.shape[0], k, nprobe, rerank,
               None if d_bitmap is None else d_bitmap.data_ptr(), d_ids.data_ptr(), d_dist.data_ptr(),
               d_lens.data_ptr(), stream)

    def search_sharded_device(self, d_queries, k: int, nprobe: int, rerank: int, d_ids, d_dist, d_lens, stream: int,
                              d_bitmap=None) -> None:
        """The row-sharded search (pxc_ivfpq_search_sharded): this rank's shard, the library's exchange,
        the global top-k on every rank. The context must have joined the communicator."""
        N.call("pxc_ivfpq_search_sharded", self.handle, d_queries.data_ptr(), d_queries.shape[0], k, nprobe,
               rerank, None if d_bitmap is None else d_bitmap.data_ptr(), d_ids.data_ptr(), d_dist.data_ptr(),
               d_lens.data_ptr(), stream)

    def last_scan_ms(self) -> float:
        return N.load().pxc_ivfpq_last_scan_ms(self.handle)

    def last_scanned(self) -> int:
        return N.load().pxc_ivfpq_last_scanned(self.handle)
