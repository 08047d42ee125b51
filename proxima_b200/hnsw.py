"""The exhaustive filtered scan of HnswIndex on the GPU.

HnswIndex's graph walk is pointer chasing and stays on the host; what moves to
the device is its fallback: when the filter is so selective that the escalating
traversal cannot gather enough accepted nodes, the reference scans the whole
store (crates/proxima-index/src/hnsw.rs:1120-1143 decides, :1189-1198 scans:
every live slot in slot order, `filter.accepts`, `space.distance`, TopK), which is
FlatIndex::search's loop over the HNSW store. ``HnswStoreMirror`` keeps that
store on the device (``pxc_flat_*``): rows, ids and liveness, with the HNSW
store's removal rule (a removed id's slot is detached, not freed: the graph
still has edges into it, so it is never handed to a later insert), and answers
``exhaustive`` with the flat kernels; a MetadataFilter is evaluated on the
device (typed filter pushdown).
"""
from __future__ import annotations

from .errors import UnknownId
from .index import AcceptAll, FlatIndex


class HnswStoreMirror(FlatIndex):
    """The device side of an HnswIndex's VectorStore, for the exhaustive fallback."""

    def remove(self, id: int) -> None:
        """VectorStore::detach: the id leaves, the slot stays reserved (tombstoned)."""
        id = int(id)
        slot = self._by_id.pop(id, None)
        if slot is None:
            raise UnknownId(id)
        self._live[slot] = 0
        self._meta[slot] = dict()
        self._meta_version += 1
        self._mark(slot, slot + 1)

    def exhaustive(self, query, k: int, filter=AcceptAll):
        """HnswIndex::exhaustive (hnsw.rs:1189-1198) for one query."""
        return self.search(query, k, filter)

    def exhaustive_batch(self, queries, k: int, filter=AcceptAll):
        """The same for a batch of queries (one device search)."""
        return self.search_batch(queries, k, filter)
