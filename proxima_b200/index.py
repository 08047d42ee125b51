"""Host mirror of proxima-index's VectorIndex contract over the B200 backend.

``FlatIndex`` keeps the reference's VectorStore semantics on the host (slot
array, LIFO slot reuse, id -> slot map, metadata; crates/proxima-core/src/storage.rs
and id.rs:137-229) and keeps a device mirror of the rows in sync through
``pxc_flat_sync``. ``search`` / ``search_batch`` evaluate the filter closure
once per live slot into a bitmap, exactly where the reference calls
``filter.accepts`` inside the scan (crates/proxima-index/src/flat.rs:162-167),
and run the scan on the GPU. Results are identical to the reference's.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field
from typing import Callable, Iterable

import numpy as np

from . import _native as N
from .core import MAX_K, Metric, SearchResult, VectorSpace
from .errors import Configuration, DuplicateId, UnknownId

Metadata = dict
Filter = Callable[[int, dict], bool]


class _AcceptAll:
    """crates/proxima-index/src/index.rs:43-50."""

    def __call__(self, _id: int, _meta: dict) -> bool:
        return True

    accepts = __call__


AcceptAll = _AcceptAll()


def check_k(k: int) -> None:
    """crates/proxima-index/src/index.rs:212-224."""
    if k > MAX_K or k < 0:
        raise Configuration("k", k, "exceeds the 16777216 result ceiling")


class Context:
    """One CUDA device (pxc_ctx). One context per process and GPU."""

    _default: dict[int, "Context"] = {}

    def __init__(self, device: int = 0):
        lib = N.load()
        self._lib = lib
        self.device = device
        dev = (C.c_int * 1)(device)
        handle = N.vp()
        N.call("pxc_ctx_create", dev, 1, C.byref(handle))
        self.handle = handle

    @classmethod
    def default(cls, device: int = 0) -> "Context":
        if device not in cls._default:
            cls._default[device] = Context(device)
        return cls._default[device]

    def set_wait_limit(self, ms: int) -> None:
        N.call("pxc_ctx_set_wait_limit", self.handle, ms)

    def set_option(self, name: str, value: int) -> None:
        """A diagnostic switch of the native library (tests only; see pxc_ctx_set_option)."""
        N.call("pxc_ctx_set_option", self.handle, name.encode(), int(value))

    def close(self) -> None:
        if getattr(self, "handle", None):
            self._lib.pxc_ctx_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


@dataclass
class IndexStats:
    """crates/proxima-index/src/index.rs:68-130."""

    len: int
    deleted: int
    dim: int
    metric: Metric
    layers: int
    nodes_per_layer: list
    edges: int
    vector_bytes: int
    graph_bytes: int

    def mean_degree(self) -> float:
        n = self.len + self.deleted
        return 0.0 if n == 0 else float(np.float32(self.edges) / np.float32(n))

    def total_bytes(self) -> int:
        return self.vector_bytes + self.graph_bytes

    def bytes_per_vector(self) -> float:
        return 0.0 if self.len == 0 else float(np.float32(self.total_bytes()) / np.float32(self.len))


class FlatIndex:
    """FlatIndex (crates/proxima-index/src/flat.rs) backed by pxc_flat."""

    def __init__(self, space: VectorSpace, ctx: Context | None = None, capacity: int = 0):
        self.space = space
        self.ctx = ctx or Context.default()
        self._lib = N.load()
        cap = max(int(capacity), 16)
        self._rows = np.zeros((cap, space.dim), dtype=np.float32)
        self._ids = np.zeros(cap, dtype=np.uint64)
        self._live = np.zeros(cap, dtype=np.uint8)
        self._meta: list[dict] = [dict() for _ in range(cap)]
        self._next = 0          # SlotAllocator.next (high-water mark)
        self._free: list[int] = []  # SlotAllocator.free (LIFO)
        self._by_id: dict[int, int] = {}
        self._dirty_lo = None
        self._dirty_hi = 0
        self._synced_hw = 0
        handle = N.vp()
        N.call("pxc_flat_create", self.ctx.handle, space.dim, int(space.metric), C.byref(handle))
        self.handle = handle
        # device columns of the metadata fields MetadataFilters read (typed filter pushdown)
        self._columns = None
        self._meta_version = 0
        self._col_version: dict[str, tuple[int, int]] = {}

    # ---- construction helpers (flat.rs:216-236) ----
    @classmethod
    def from_array(cls, space: VectorSpace, data, ctx: Context | None = None) -> "FlatIndex":
        """TryFrom<(&VectorSpace, &[f32])>: ids 0..n in order; rows prepared."""
        a = np.asarray(data, dtype=np.float32)
        if a.ndim == 1:
            if a.size % space.dim != 0:
                raise Configuration("data", a.size, "must be a multiple of the space dimension")
            a = a.reshape(-1, space.dim)
        n = a.shape[0]
        idx = cls(space, ctx, capacity=n)
        prepared = space.prepare_batch(a)
        idx._rows[:n] = prepared
        idx._ids[:n] = np.arange(n, dtype=np.uint64)
        idx._live[:n] = 1
        idx._by_id = {i: i for i in range(n)}
        idx._next = n
        idx._mark(0, n)
        return idx

    def close(self) -> None:
        if getattr(self, "_columns", None) is not None:
            self._columns.close()
            self._columns = None
        if getattr(self, "handle", None):
            self._lib.pxc_flat_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- store plumbing ----
    def _grow(self, need: int) -> None:
        cap = self._rows.shape[0]
        if need <= cap:
            return
        ncap = max(need, cap * 2)
        rows = np.zeros((ncap, self.space.dim), dtype=np.float32)
        rows[:cap] = self._rows
        ids = np.zeros(ncap, dtype=np.uint64)
        ids[:cap] = self._ids
        live = np.zeros(ncap, dtype=np.uint8)
        live[:cap] = self._live
        self._rows, self._ids, self._live = rows, ids, live
        self._meta.extend(dict() for _ in range(ncap - cap))

    def _mark(self, lo: int, hi: int) -> None:
        self._dirty_lo = lo if self._dirty_lo is None else min(self._dirty_lo, lo)
        self._dirty_hi = max(self._dirty_hi, hi)

    def _allocate(self) -> int:
        if self._free:
            return self._free.pop()
        slot = self._next
        self._next += 1
        self._grow(self._next)
        return slot

    def _sync(self) -> None:
        if self._next < self._synced_hw:
            N.call("pxc_flat_truncate", self.handle, self._next)
            self._synced_hw = self._next
        if self._dirty_lo is None:
            return
        lo, hi = self._dirty_lo, min(self._dirty_hi, self._next)
        lo = min(lo, self._synced_hw)  # the mirror may not have gaps
        if hi > lo:
            N.call("pxc_flat_sync", self.handle, N.ptr(self._rows[lo:hi]), N.ptr(self._ids[lo:hi]),
                   N.ptr(self._live[lo:hi]), lo, hi - lo)
        self._synced_hw = max(self._synced_hw, hi)
        self._dirty_lo, self._dirty_hi = None, 0

    # ---- VectorIndex (crates/proxima-index/src/index.rs:154-205) ----
    def insert(self, id: int, vector, metadata: dict | None = None) -> None:
        prepared = self.space.prepare(vector)
        id = int(id)
        if id in self._by_id:
            raise DuplicateId(id)
        slot = self._allocate()
        self._rows[slot] = prepared
        self._ids[slot] = id
        self._live[slot] = 1
        self._meta[slot] = dict(metadata or {})
        self._meta_version += 1
        self._by_id[id] = slot
        self._mark(slot, slot + 1)

    def remove(self, id: int) -> None:
        id = int(id)
        slot = self._by_id.pop(id, None)
        if slot is None:
            raise UnknownId(id)
        self._live[slot] = 0
        self._meta[slot] = dict()
        self._meta_version += 1
        self._free.append(slot)
        self._mark(slot, slot + 1)

    def upsert(self, id: int, vector, metadata: dict | None = None) -> None:
        if self.contains(id):
            self.remove(id)
        self.insert(id, vector, metadata)

    def contains(self, id: int) -> bool:
        return int(id) in self._by_id

    def __len__(self) -> int:
        return len(self._by_id)

    def len(self) -> int:
        return len(self._by_id)

    def is_empty(self) -> bool:
        return not self._by_id

    def vector(self, id: int):
        slot = self._by_id.get(int(id))
        return None if slot is None else self._rows[slot].copy()

    def metadata(self, id: int):
        slot = self._by_id.get(int(id))
        return None if slot is None else self._meta[slot]

    def set_metadata(self, id: int, metadata: dict) -> None:
        slot = self._by_id.get(int(id))
        if slot is None:
            raise UnknownId(int(id))
        self._meta[slot] = dict(metadata)
        self._meta_version += 1

    def ids(self) -> list[int]:
        return [int(self._ids[s]) for s in range(self._next) if self._live[s]]

    def clear(self) -> None:
        self._meta_version += 1
        self._live[: self._next] = 0
        self._next = 0
        self._free.clear()
        self._by_id.clear()
        self._dirty_lo, self._dirty_hi = None, 0

    def stats(self) -> IndexStats:
        return IndexStats(len=len(self), deleted=0, dim=self.space.dim, metric=self.space.metric,
                          layers=1, nodes_per_layer=[len(self)], edges=0,
                          vector_bytes=self._rows.shape[0] * self.space.dim * 4, graph_bytes=0)

    def _bitmap(self, filter) -> np.ndarray | None:
        if filter is None or filter is AcceptAll or isinstance(filter, _AcceptAll):
            return None
        accepts = getattr(filter, "accepts", filter)
        words = np.zeros((self._next + 63) // 64, dtype=np.uint64)
        bits = np.zeros(self._next, dtype=bool)
        for s in range(self._next):
            if self._live[s] and accepts(int(self._ids[s]), self._meta[s]):
                bits[s] = True
        if self._next:
            packed = np.packbits(bits, bitorder="little")
            packed = np.concatenate([packed, np.zeros(words.size * 8 - packed.size, dtype=np.uint8)])
            words[:] = packed.view(np.uint64)
        return words

    def _device_columns(self, flt) -> "DeviceColumns":
        """The device columns of the fields `flt` reads, re-uploaded when the metadata changed."""
        from .filters import DeviceColumns

        if self._columns is None:
            self._columns = DeviceColumns(self.ctx)
        for field in flt.fields():
            if self._col_version.get(field) != (self._meta_version, self._next):
                vals = [self._meta[s].get(field) if self._live[s] else None for s in range(self._next)]
                self._columns.set_values(field, vals, 0)
                self._columns.truncate(self._next)
                self._col_version[field] = (self._meta_version, self._next)
        return self._columns

    def search_where_prepared(self, prepared: np.ndarray, k: int, flt):
        """Batched search with a MetadataFilter evaluated on the device (pxc_flat_search_where)."""
        check_k(k)
        self._sync()
        cols = self._device_columns(flt)
        conds, nc, ops, no = flt.compile(cols)
        nq = prepared.shape[0]
        ids = np.zeros((nq, max(k, 1)), dtype=np.uint64)
        dist = np.zeros((nq, max(k, 1)), dtype=np.float32)
        lens = np.zeros(nq, dtype=np.uint32)
        if nq:
            N.call("pxc_flat_search_where", self.handle, cols.handle, conds, nc, ops, no, N.ptr(prepared), nq, k,
                   N.ptr(ids), N.ptr(dist), N.ptr(lens))
        return ids[:, :k], dist[:, :k], lens

    def search_prepared_batch(self, prepared: np.ndarray, k: int, bitmap: np.ndarray | None = None):
        """Batched search of already-prepared [nq, dim] queries; returns (ids, dist, lens)."""
        check_k(k)
        self._sync()
        nq = prepared.shape[0]
        ids = np.zeros((nq, max(k, 1)), dtype=np.uint64)
        dist = np.zeros((nq, max(k, 1)), dtype=np.float32)
        lens = np.zeros(nq, dtype=np.uint32)
        if nq:
            N.call("pxc_flat_search", self.handle, N.ptr(prepared), nq, k, N.ptr(bitmap),
                   N.ptr(ids), N.ptr(dist), N.ptr(lens))
        return ids[:, :k], dist[:, :k], lens

    def search_batch(self, queries, k: int, filter=AcceptAll) -> list[list[SearchResult]]:
        """search for every query of a flat or 2-D array (the batched trait method). A MetadataFilter
        is evaluated on the device; any other filter closure once per live slot on the host."""
        from .filters import MetadataFilter

        check_k(k)
        prepared = self.space.prepare_batch(queries)
        if isinstance(filter, MetadataFilter):
            ids, dist, lens = self.search_where_prepared(prepared, k, filter)
        else:
            ids, dist, lens = self.search_prepared_batch(prepared, k, self._bitmap(filter))
        return [[SearchResult(int(ids[q, i]), float(dist[q, i])) for i in range(int(lens[q]))]
                for q in range(prepared.shape[0])]

    def search(self, query, k: int, filter=AcceptAll) -> list[SearchResult]:
        from .filters import MetadataFilter

        check_k(k)
        prepared = self.space.prepare(query)[None, :]
        if isinstance(filter, MetadataFilter):
            ids, dist, lens = self.search_where_prepared(prepared, k, filter)
        else:
            ids, dist, lens = self.search_prepared_batch(prepared, k, self._bitmap(filter))
        return [SearchResult(int(ids[0, i]), float(dist[0, i])) for i in range(int(lens[0]))]

    def search_all(self, query, k: int) -> list[SearchResult]:
        return self.search(query, k, AcceptAll)

    def exact_ids(self, query, k: int, filter=AcceptAll) -> list[int]:
        return [h.id for h in self.search(query, k, filter)]

    def device_path(self) -> int:
        """1 if the next search runs the tensor-core u8 scan, 0 for the fp32 scan."""
        self._sync()
        return int(self._lib.pxc_flat_path(self.handle))

    def last_redone(self) -> int:
        """Queries of the last search that the first tensor-core pass did not settle and that were
        answered again (see pxc_flat_last_redone)."""
        return int(self._lib.pxc_flat_last_redone(self.handle))


@dataclass
class RecallReport:
    """crates/proxima-index/src/recall.rs:27-56."""

    queries: int
    k: int
    mean: float
    min: float
    per_query: list = field(default_factory=list)
    short_results: int = 0

    def below(self, threshold: float) -> float:
        if not self.per_query:
            return 0.0
        return float(np.float32(sum(1 for r in self.per_query if r < threshold)) /
                     np.float32(len(self.per_query)))


def _overlap(exact: list[int], approx: list[SearchResult]) -> float:
    """recall.rs:176-187."""
    if not exact:
        return 1.0
    s = set(exact)
    hits = sum(1 for h in approx if h.id in s)
    return float(np.float32(hits) / np.float32(len(exact)))


def recall_at_k(candidate, truth: FlatIndex, queries, k: int, filter=AcceptAll) -> RecallReport:
    """recall_at_k[_filtered] (crates/proxima-index/src/recall.rs:108-169), batched on the GPU."""
    dim = truth.space.dim
    q = np.asarray(queries, dtype=np.float32).reshape(-1)
    if dim == 0 or q.size % dim != 0:  # recall.rs:131-137
        raise Configuration("queries", q.size, "must be a multiple of the index dimension")
    if q.size == 0:
        return RecallReport(0, k, 0.0, 0.0, [], 0)
    exact = truth.search_batch(q, k, filter)
    approx = candidate.search_batch(q, k, filter)
    per_query, short = [], 0
    for e, a in zip(exact, approx):
        if len(a) < len(e):
            short += 1
        per_query.append(_overlap([h.id for h in e], a))
    # recall.rs:155: Iterator::sum over f32 is a sequential fold, then one division
    total = np.float32(0.0)
    for r in per_query:
        total = np.float32(total + np.float32(r))
    mean = float(total / np.float32(len(per_query)))
    mn = min(per_query)
    return RecallReport(len(per_query), k, mean, mn, per_query, short)
