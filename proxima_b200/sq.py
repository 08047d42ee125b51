"""Host mirror of proxima-quantize's ScalarQuantizer and the SQ filtered search.

``ScalarQuantizer`` keeps the reference's interface
(crates/proxima-quantize/src/scalar.rs: ``train(space, training, mode, code_type)``,
``encode`` / ``encode_into``, ``decode``, the range table) and runs on the GPU
through ``pxc_sq_*``; there is no CPU path.

``SqIndex`` is the new composition the scalar-quantized filtered scan needs
(the reference has no SQ index): a store of prepared vectors with their I8
codes and integer metadata columns, searched as an int8 over-fetch on the
tensor cores followed by an exact re-rank (``pxc_sq_search``).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from enum import IntEnum

import numpy as np

from . import _native as N
from .core import Metric


class RangeMode(IntEnum):
    """crates/proxima-quantize/src/scalar.rs RangeMode."""

    GLOBAL = 0
    PER_DIMENSION = 1


class CodeType(IntEnum):
    """crates/proxima-quantize/src/scalar.rs CodeType."""

    U8 = 0
    I8 = 1


INT64_MAX = (1 << 63) - 1
INT64_MIN = -(1 << 63)


@dataclass
class IntRange:
    """``lo <= metadata[column] <= hi`` (a typed Int filter condition)."""

    column: int
    lo: int = INT64_MIN
    hi: int = INT64_MAX


def _is_cuda(x) -> bool:
    return hasattr(x, "is_cuda") and x.is_cuda


class ScalarQuantizer:
    """ScalarQuantizer (scalar.rs:111-123): ``min``, ``scale`` and
    ``inverse_scale`` per group (one group under GLOBAL, ``dim`` under
    PER_DIMENSION)."""

    def __init__(self, dim: int, mode: RangeMode, code_type: CodeType, min_, scale, inverse_scale, context=None):
        from .index import Context

        self.ctx = context or Context.default()
        self.dim = dim
        self.mode = RangeMode(mode)
        self.code_type = CodeType(code_type)
        self.min = np.ascontiguousarray(min_, np.float32)
        self.scale = np.ascontiguousarray(scale, np.float32)
        self.inverse_scale = np.ascontiguousarray(inverse_scale, np.float32)

    @property
    def groups(self) -> int:
        return 1 if self.mode == RangeMode.GLOBAL else self.dim

    @classmethod
    def train(cls, dim: int, training, mode: RangeMode = RangeMode.PER_DIMENSION,
              code_type: CodeType = CodeType.U8, context=None) -> "ScalarQuantizer":
        """scalar.rs:141-195. ``training`` is a flat or (n, dim) float32 array
        on the host or a CUDA torch tensor."""
        from .index import Context

        ctx = context or Context.default()
        groups = 1 if RangeMode(mode) == RangeMode.GLOBAL else dim
        mn = np.zeros(groups, np.float32)
        sc = np.zeros(groups, np.float32)
        inv = np.zeros(groups, np.float32)
        if _is_cuda(training):
            import torch

            t = training.contiguous().view(-1)
            if t.numel() == 0 or t.numel() % dim:
                n = 0
            else:
                n = t.numel() // dim
            N.call("pxc_sq_train_device", ctx.handle, t.data_ptr(), n, dim, int(mode), N.ptr(mn), N.ptr(sc),
                   N.ptr(inv), torch.cuda.current_stream(t.device).cuda_stream)
        else:
            t = np.ascontiguousarray(training, np.float32).reshape(-1)
            n = t.size // dim if (t.size and t.size % dim == 0) else 0
            N.call("pxc_sq_train", ctx.handle, N.ptr(t) if t.size else None, n, dim, int(mode), N.ptr(mn),
                   N.ptr(sc), N.ptr(inv))
        return cls(dim, mode, code_type, mn, sc, inv, ctx)

    def encode(self, vectors):
        """encode_into (scalar.rs:246-268) for every row; host array or CUDA tensor in, same kind out."""
        if _is_cuda(vectors):
            import torch

            v = vectors.contiguous().view(-1, self.dim)
            out = torch.empty((v.shape[0], self.dim), dtype=torch.uint8, device=v.device)
            N.call("pxc_sq_encode_device", self.ctx.handle, N.ptr(self.min), N.ptr(self.inverse_scale), self.dim,
                   int(self.mode), int(self.code_type), v.data_ptr(), v.shape[0], out.data_ptr(),
                   torch.cuda.current_stream(v.device).cuda_stream)
            return out
        v = np.ascontiguousarray(vectors, np.float32).reshape(-1, self.dim)
        out = np.zeros((v.shape[0], self.dim), np.uint8)
        N.call("pxc_sq_encode", self.ctx.handle, N.ptr(self.min), N.ptr(self.inverse_scale), self.dim,
               int(self.mode), int(self.code_type), N.ptr(v), v.shape[0], N.ptr(out))
        return out

    def asymmetric(self, queries, codes, metric: Metric = Metric.EUCLIDEAN) -> np.ndarray:
        """asymmetric_squared_l2 (EUCLIDEAN) or asymmetric_inner_product (INNER_PRODUCT, COSINE on
        prepared vectors), scalar.rs:298-327, for every (query, code) pair: an (nq, n) float32 array."""
        q = np.ascontiguousarray(queries, np.float32).reshape(-1, self.dim)
        c = np.ascontiguousarray(codes, np.uint8).reshape(-1, self.dim)
        out = np.zeros((q.shape[0], c.shape[0]), np.float32)
        N.call("pxc_sq_asymmetric", self.ctx.handle, N.ptr(self.min), N.ptr(self.scale), self.dim,
               int(self.mode), int(self.code_type), int(metric), N.ptr(q), q.shape[0], N.ptr(c), c.shape[0],
               N.ptr(out))
        return out

    def asymmetric_squared_l2(self, query, code) -> float:
        """scalar.rs:298-305 for one query and one code."""
        return float(self.asymmetric(query, code, Metric.EUCLIDEAN)[0, 0])

    def asymmetric_inner_product(self, query, code) -> float:
        """scalar.rs:313-319 for one query and one code."""
        return float(self.asymmetric(query, code, Metric.INNER_PRODUCT)[0, 0])

    def decode(self, codes) -> np.ndarray:
        """decode (scalar.rs:270-296): min + level * scale per component."""
        c = np.ascontiguousarray(codes, np.uint8).reshape(-1, self.dim)
        out = np.zeros((c.shape[0], self.dim), np.float32)
        N.call("pxc_sq_decode", self.ctx.handle, N.ptr(self.min), N.ptr(self.scale), self.dim, int(self.mode),
               int(self.code_type), N.ptr(c), c.shape[0], N.ptr(out))
        return out


def combine_ranges(per_rank_min, per_rank_max):
    """Fold per-rank (min, max) tables in rank order with the reference's strict
    comparisons (``v < min`` / ``v > max``): the single-pass result over the
    concatenated training rows. Returns (min, scale, inverse_scale) in f32."""
    mn = np.array(per_rank_min[0], np.float32)
    mx = np.array(per_rank_max[0], np.float32)
    for lo, hi in zip(per_rank_min[1:], per_rank_max[1:]):
        lo = np.asarray(lo, np.float32)
        hi = np.asarray(hi, np.float32)
        mn = np.where(lo < mn, lo, mn)
        mx = np.where(hi > mx, hi, mx)
    scale = ((mx - mn) / np.float32(255.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(scale > 0, np.float32(1.0) / np.where(scale > 0, scale, np.float32(1.0)), np.float32(0.0))
    return mn, scale, inv.astype(np.float32)


def ranges_device(training, dim: int, mode: RangeMode = RangeMode.PER_DIMENSION, context=None):
    """Observed (min, max) per group of a CUDA tensor of training rows."""
    import torch

    from .index import Context

    ctx = context or Context.default()
    groups = 1 if RangeMode(mode) == RangeMode.GLOBAL else dim
    lo = np.zeros(groups, np.float32)
    hi = np.zeros(groups, np.float32)
    t = training.contiguous().view(-1)
    N.call("pxc_sq_ranges_device", ctx.handle, t.data_ptr(), t.numel() // dim, dim, int(mode), N.ptr(lo), N.ptr(hi),
           torch.cuda.current_stream(t.device).cuda_stream)
    return lo, hi


class SqIndex:
    """Scalar-quantized filtered index: int8 over-fetch, exact re-rank."""

    def __init__(self, dim: int, metric: Metric = Metric.COSINE, context=None):
        from .index import Context

        self.ctx = context or Context.default()
        self.dim = dim
        self.metric = Metric(metric)
        h = N.vp()
        N.call("pxc_sq_create", self.ctx.handle, dim, int(self.metric), C.byref(h))
        self.handle = h
        self.nslots = 0

    def close(self) -> None:
        if getattr(self, "handle", None):
            N.load().pxc_sq_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_store(self, vectors, ids=None, live=None) -> None:
        """Prepared vectors per slot (host array or CUDA tensor), VectorIds, live flags."""
        i = None if ids is None else np.ascontiguousarray(ids, np.uint64)
        lv = None if live is None else np.ascontiguousarray(live, np.uint8)
        if _is_cuda(vectors):
            v = vectors.contiguous()
            n = v.numel() // self.dim
            N.call("pxc_sq_set_store_device", self.handle, v.data_ptr(), N.ptr(i), N.ptr(lv), n)
        else:
            v = np.ascontiguousarray(vectors, np.float32).reshape(-1, self.dim)
            n = v.shape[0]
            N.call("pxc_sq_set_store", self.handle, N.ptr(v), N.ptr(i), N.ptr(lv), n)
        self.nslots = n

    def set_quantizer(self, sq: ScalarQuantizer) -> None:
        N.call("pxc_sq_set_quantizer", self.handle, int(sq.mode), N.ptr(sq.min), N.ptr(sq.scale),
               N.ptr(sq.inverse_scale))

    def train(self, mode: RangeMode = RangeMode.PER_DIMENSION) -> ScalarQuantizer:
        """ScalarQuantizer::train over the live stored rows, then encode them."""
        N.call("pxc_sq_train_store", self.handle, int(mode))
        return self.quantizer()

    def quantizer(self) -> ScalarQuantizer:
        mode = C.c_int32()
        N.call("pxc_sq_get_quantizer", self.handle, C.byref(mode), None, None, None)
        groups = 1 if mode.value == RangeMode.GLOBAL else self.dim
        mn = np.zeros(groups, np.float32)
        sc = np.zeros(groups, np.float32)
        inv = np.zeros(groups, np.float32)
        N.call("pxc_sq_get_quantizer", self.handle, None, N.ptr(mn), N.ptr(sc), N.ptr(inv))
        return ScalarQuantizer(self.dim, RangeMode(mode.value), CodeType.I8, mn, sc, inv, self.ctx)

    def set_column(self, column: int, values, present=None) -> None:
        v = np.ascontiguousarray(values, np.int64)
        p = None if present is None else np.ascontiguousarray(present, np.uint8)
        N.call("pxc_sq_set_column", self.handle, column, N.ptr(v), N.ptr(p))

    def __len__(self) -> int:
        return int(N.load().pxc_sq_len(self.handle))

    def codes(self) -> np.ndarray:
        """The stored I8 codes per slot (dead slots zero)."""
        out = np.zeros((max(self.nslots, 1), self.dim), np.uint8)
        N.call("pxc_sq_get_codes", self.handle, N.ptr(out))
        return out[:self.nslots]

    @staticmethod
    def _ranges(ranges):
        rs = list(ranges or [])
        if not rs:
            return None, 0
        arr = (N.PxcIntRange * len(rs))()
        for j, r in enumerate(rs):
            arr[j].column, arr[j].reserved, arr[j].lo, arr[j].hi = r.column, 0, r.lo, r.hi
        return arr, len(rs)

    def search_batch(self, queries, k: int, overfetch: int = 100, bitmap=None, ranges=None):
        """(ids, distances, lengths) for a batch of prepared queries."""
        q = np.ascontiguousarray(queries, np.float32).reshape(-1, self.dim)
        nq = len(q)
        kk = max(k, 1)
        ids = np.zeros((nq, kk), np.uint64)
        dist = np.zeros((nq, kk), np.float32)
        lens = np.zeros(nq, np.uint32)
        bm = None if bitmap is None else np.ascontiguousarray(bitmap, np.uint64)
        arr, nr = self._ranges(ranges)
        N.call("pxc_sq_search", self.handle, N.ptr(q), nq, k, overfetch, N.ptr(bm), arr, nr, N.ptr(ids),
               N.ptr(dist), N.ptr(lens))
        return ids[:, :k], dist[:, :k], lens

    def search_device(self, d_queries, k: int, overfetch: int, d_ids, d_dist, d_lens, stream: int, d_bitmap=None,
                      ranges=None) -> None:
        """Device-buffer search (torch tensors) on `stream`; returns when done."""
        arr, nr = self._ranges(ranges)
        N.call("pxc_sq_search_device", self.handle, d_queries.data_ptr(), d_queries.shape[0], k, overfetch,
               None if d_bitmap is None else d_bitmap.data_ptr(), arr, nr, d_ids.data_ptr(), d_dist.data_ptr(),
               d_lens.data_ptr(), stream)

    def last_scan_ms(self) -> float:
        return N.load().pxc_sq_last_scan_ms(self.handle)

    def last_accepted(self) -> int:
        return int(N.load().pxc_sq_last_accepted(self.handle))

    def last_fallback(self) -> int:
        return int(N.load().pxc_sq_last_fallback(self.handle))

    def last_retried(self) -> int:
        return int(N.load().pxc_sq_last_retried(self.handle))
