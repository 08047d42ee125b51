"""Host-side mirror of proxima-core's types: Metric, VectorSpace, SearchResult.

``VectorSpace.prepare`` reproduces crates/proxima-core/src/space.rs:130-138 and
distance.rs:508-517 operation for operation (eight lane accumulators, pairwise
reduce, tail, sqrt, one reciprocal, multiply), in float32 numpy arithmetic,
which rounds each operation as IEEE single precision does and never fuses.
"""
from __future__ import annotations

import enum
from dataclasses import dataclass

import numpy as np

from .errors import Configuration, DimensionMismatch, NonFinite

MAX_DIM = 1 << 20  # space.rs: MAX_DIM
MAX_K = 1 << 24    # index.rs:212-224 check_k


class Metric(enum.IntEnum):
    """crates/proxima-core/src/distance.rs:90-135 (same order as the C ABI codes)."""

    EUCLIDEAN = 0
    COSINE = 1
    INNER_PRODUCT = 2
    MANHATTAN = 3

    def requires_normalization(self) -> bool:
        return self is Metric.COSINE

    def is_true_metric(self) -> bool:
        return self in (Metric.EUCLIDEAN, Metric.MANHATTAN)

    def to_true_distance(self, score: float) -> float:
        if self is Metric.EUCLIDEAN:
            return float(np.sqrt(np.float32(score)))
        if self is Metric.INNER_PRODUCT:
            return -score
        return score

    @staticmethod
    def from_name(name: str) -> "Metric | None":
        return {"euclidean": Metric.EUCLIDEAN, "cosine": Metric.COSINE,
                "inner_product": Metric.INNER_PRODUCT, "manhattan": Metric.MANHATTAN}.get(name)

    def __str__(self) -> str:
        return self.name.lower()


@dataclass(frozen=True)
class SearchResult:
    """crates/proxima-core/src/topk.rs:33-67: ordered by (total_cmp(distance), id)."""

    id: int
    distance: float


def dot8_rows(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """dot_unrolled (distance.rs:317-331) for each row pair of two [n, dim] f32 arrays."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    n, dim = a.shape
    full = dim // 8 * 8
    acc = np.zeros((n, 8), dtype=np.float32)
    for g in range(0, full, 8):
        acc = acc + a[:, g:g + 8] * b[:, g:g + 8]
    tail = np.zeros(n, dtype=np.float32)
    for i in range(full, dim):
        tail = tail + a[:, i] * b[:, i]
    lo = (acc[:, 0] + acc[:, 1]) + (acc[:, 2] + acc[:, 3])
    hi = (acc[:, 4] + acc[:, 5]) + (acc[:, 6] + acc[:, 7])
    return (lo + hi) + tail


def normalize_rows(rows: np.ndarray) -> np.ndarray:
    """normalize_in_place (distance.rs:508-517) on every row, in place; returns the norms."""
    norms = np.sqrt(dot8_rows(rows, rows))
    ok = (norms > 0) & np.isfinite(norms)
    if ok.any():
        inv = np.float32(1.0) / norms[ok]
        rows[ok] = rows[ok] * inv[:, None]
    return norms


class VectorSpace:
    """crates/proxima-core/src/space.rs:54-156."""

    def __init__(self, dim: int, metric: Metric):
        if dim < 1:
            raise Configuration("dim", dim, "must be at least 1; a 0-dimensional space makes all distances equal")
        if dim > MAX_DIM:
            raise Configuration("dim", dim, "exceeds the 1048576 dimension ceiling")
        self.dim = int(dim)
        self.metric = Metric(metric)

    def validate(self, vector) -> np.ndarray:
        v = np.asarray(vector, dtype=np.float32)
        if v.ndim != 1 or v.shape[0] != self.dim:
            raise DimensionMismatch(self.dim, int(v.size))
        bad = np.flatnonzero(~np.isfinite(v))
        if bad.size:
            raise NonFinite(int(bad[0]), float(v[bad[0]]))
        return v

    def prepare(self, vector) -> np.ndarray:
        """Validate, and for cosine return a normalised copy (Cow::Owned)."""
        v = self.validate(vector)
        if not self.metric.requires_normalization():
            return v
        out = v.copy()[None, :]
        normalize_rows(out)
        return out[0]

    def prepare_batch(self, flat) -> np.ndarray:
        """prepare for a flat [n*dim] (or [n, dim]) query array; returns [n, dim] f32."""
        a = np.asarray(flat, dtype=np.float32)
        if a.ndim == 1:
            if a.size % self.dim != 0:
                raise Configuration("queries", a.size, "must be a multiple of the index dimension")
            a = a.reshape(-1, self.dim)
        elif a.ndim != 2 or a.shape[1] != self.dim:
            raise DimensionMismatch(self.dim, int(a.shape[-1]) if a.ndim else 0)
        if not np.isfinite(a).all():
            bad = int(np.flatnonzero(~np.isfinite(a.reshape(-1)))[0])
            raise NonFinite(bad % self.dim, float(a.reshape(-1)[bad]))
        a = np.ascontiguousarray(a, dtype=np.float32)
        if self.metric.requires_normalization():
            a = a.copy()
            normalize_rows(a)
        return a

    def vector_bytes(self) -> int:
        return self.dim * 4

    def __str__(self) -> str:
        return f"{self.dim}d/{self.metric}"
