"""ctypes wrapper of the CPU oracle (oracle/lib/liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU legs of bench.py (cpu_baseline and --impl reference), as the checker or
the timed CPU baseline. The product path never imports it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "lib" / "liboracle.so"

EUCLIDEAN, COSINE, INNER_PRODUCT, MANHATTAN = 0, 1, 2, 3
RANGE_GLOBAL, RANGE_PER_DIMENSION = 0, 1
CODE_U8, CODE_I8 = 0, 1

_lib = None
vp, u64, i64, f32, f64, i32 = C.c_void_p, C.c_uint64, C.c_int64, C.c_float, C.c_double, C.c_int


class Rng(C.Structure):
    _fields_ = [("key", C.c_uint32 * 8), ("counter", C.c_uint64), ("buf", C.c_uint32 * 64),
                ("index", C.c_uint32)]


class IvfReport(C.Structure):
    _fields_ = [("sampled", u64), ("coarse_iterations", u64), ("populated_lists", u64),
                ("largest_list", u64), ("produced", u64), ("coarse_inertia", f64),
                ("residual_inertia", f64)]


def build() -> Path:
    if not LIB.exists() or LIB.stat().st_mtime < (HERE / "pxo.cpp").stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


def lib():
    global _lib
    if _lib is None:
        build()
        L = C.CDLL(str(LIB))
        sig = {
            "pxo_squared_euclidean": (f32, [vp, vp, u64]),
            "pxo_squared_euclidean_scalar": (f32, [vp, vp, u64]),
            "pxo_dot": (f32, [vp, vp, u64]),
            "pxo_manhattan": (f32, [vp, vp, u64]),
            "pxo_cosine": (f32, [vp, vp, u64]),
            "pxo_cosine_normalized": (f32, [vp, vp, u64]),
            "pxo_normalize_in_place": (f32, [vp, u64]),
            "pxo_space_distance": (f32, [i32, vp, vp, u64]),
            "pxo_prepare": (i64, [i32, vp, u64, u64]),
            "pxo_flat_search": (None, [vp, vp, vp, u64, u64, i32, vp, u64, u64, vp, vp, vp, vp, i32]),
            "pxo_recall_overlap": (f32, [vp, C.c_uint32, vp, C.c_uint32]),
            "pxo_chacha_block": (None, [vp, u64, u64, C.c_int, vp]),
            "pxo_rng_seed_from_u64": (None, [vp, u64]),
            "pxo_rng_next_u32": (C.c_uint32, [vp]),
            "pxo_rng_next_u64": (u64, [vp]),
            "pxo_rng_gen_range_usize": (u64, [vp, u64]),
            "pxo_rng_gen_range_f64": (f64, [vp, f64, f64]),
            "pxo_kmeans": (u64, [vp, u64, u64, u64, u64, vp, u64, vp, vp, vp, vp, vp, i32]),
            "pxo_kmeans_nearest": (C.c_uint32, [vp, vp, u64, u64, vp]),
            "pxo_pq_layout": (None, [u64, u64, vp, vp]),
            "pxo_pq_train": (i32, [vp, u64, u64, u64, u64, u64, vp, vp, vp, i32]),
            "pxo_pq_encode": (None, [vp, u64, u64, vp, u64, vp]),
            "pxo_pq_decode": (None, [vp, u64, u64, vp, u64, vp]),
            "pxo_pq_distance_table": (None, [vp, u64, u64, vp, vp, vp]),
            "pxo_pq_adc_squared": (f32, [vp, u64, vp]),
            "pxo_pq_adc_inner": (f32, [vp, u64, vp]),
            "pxo_sq_train": (i64, [vp, u64, u64, i32, vp, vp, vp]),
            "pxo_sq_encode": (None, [vp, vp, u64, i32, i32, vp, u64, vp]),
            "pxo_sq_decode": (None, [vp, vp, u64, i32, i32, vp, u64, vp]),
            "pxo_sq_asymmetric_squared_l2": (f32, [vp, vp, u64, i32, i32, vp, vp]),
            "pxo_sq_asymmetric_inner_product": (f32, [vp, vp, u64, i32, i32, vp, vp]),
            "pxo_sq_query_s8": (None, [vp, u64, i32, vp, vp]),
            "pxo_sq_search": (None, [vp, u64, i32, vp, vp, vp, vp, u64, i32, vp, u64, u64, u64, vp, vp, vp, i32]),
            "pxo_ivf_nearest_centroid": (C.c_uint32, [vp, vp, u64, u64]),
            "pxo_ivfpq_train": (u64, [vp, vp, u64, u64, u64, u64, u64, u64, u64, vp, vp, vp, vp, vp,
                                      vp, vp, i32]),
            "pxo_ivfpq_encode_all": (None, [vp, vp, u64, u64, vp, u64, vp, u64, vp, vp, i32]),
            "pxo_ivfpq_search": (None, [vp, vp, vp, u64, u64, i32, vp, u64, vp, u64, vp, vp, vp, u64,
                                        u64, u64, u64, vp, vp, vp, vp, i32]),
            "pxo_crc32c_append": (C.c_uint32, [C.c_uint32, vp, u64]),
            "pxo_ivfpq_search_csr": (None, [vp, vp, vp, u64, u64, i32, vp, u64, vp, u64, vp, vp, vp, vp, u64,
                                        u64, u64, u64, vp, vp, vp, vp, i32]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data


def f32a(x) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(x, dtype=np.float32))


def threads() -> int:
    return os.cpu_count() or 1


# ---- distance.rs ----
def squared_euclidean(a, b) -> float:
    a, b = f32a(a), f32a(b)
    return lib().pxo_squared_euclidean(_p(a), _p(b), min(a.size, b.size))


def squared_euclidean_scalar(a, b) -> float:
    a, b = f32a(a), f32a(b)
    return lib().pxo_squared_euclidean_scalar(_p(a), _p(b), min(a.size, b.size))


def dot(a, b) -> float:
    a, b = f32a(a), f32a(b)
    return lib().pxo_dot(_p(a), _p(b), min(a.size, b.size))


def manhattan(a, b) -> float:
    a, b = f32a(a), f32a(b)
    return lib().pxo_manhattan(_p(a), _p(b), min(a.size, b.size))


def cosine(a, b) -> float:
    a, b = f32a(a), f32a(b)
    return lib().pxo_cosine(_p(a), _p(b), min(a.size, b.size))


def cosine_normalized(a, b) -> float:
    a, b = f32a(a), f32a(b)
    return lib().pxo_cosine_normalized(_p(a), _p(b), min(a.size, b.size))


def normalized(v) -> np.ndarray:
    v = f32a(v).copy()
    lib().pxo_normalize_in_place(_p(v), v.size)
    return v


def prepare(metric: int, rows) -> np.ndarray:
    r = f32a(rows).copy()
    if r.ndim == 1:
        r = r[None, :]
    bad = lib().pxo_prepare(metric, _p(r), r.shape[0], r.shape[1])
    if bad >= 0:
        raise ValueError(f"non-finite component {bad}")
    return r


def space_distance(metric: int, a, b) -> float:
    a, b = f32a(a), f32a(b)
    return lib().pxo_space_distance(metric, _p(a), _p(b), a.size)


# ---- flat.rs ----
def flat_search(data, queries, k: int, metric: int, ids=None, live=None, bitmap=None, nthreads=None):
    """Exact top-k of prepared queries over prepared slot-major data."""
    data, queries = f32a(data), f32a(queries)
    nslots, dim = data.shape
    nq = queries.shape[0]
    kk = max(k, 1)
    out_ids = np.zeros((nq, kk), dtype=np.uint64)
    out_d = np.zeros((nq, kk), dtype=np.float32)
    out_len = np.zeros(nq, dtype=np.uint32)
    ids = None if ids is None else np.ascontiguousarray(ids, dtype=np.uint64)
    live = None if live is None else np.ascontiguousarray(live, dtype=np.uint8)
    bitmap = None if bitmap is None else np.ascontiguousarray(bitmap, dtype=np.uint64)
    lib().pxo_flat_search(_p(data), _p(ids), _p(live), nslots, dim, metric, _p(queries), nq, k,
                          _p(bitmap), _p(out_ids), _p(out_d), _p(out_len), nthreads or threads())
    return out_ids[:, :k], out_d[:, :k], out_len


# ---- kmeans.rs ----
def kmeans(points, k: int, max_iterations: int, init=None, seed: int = 0, nthreads=None):
    pts = f32a(points)
    n, dim = pts.shape
    kk = max(min(k, n), 1)
    cent = np.zeros((kk, dim), dtype=np.float32)
    assign = np.zeros(max(n, 1), dtype=np.uint32)
    inertia = C.c_double()
    iters = C.c_uint64()
    init = None if init is None else f32a(init)
    lib().pxo_kmeans(_p(pts), n, dim, k, max_iterations, _p(init), seed, None, _p(cent),
                     _p(assign), C.byref(inertia), C.byref(iters), nthreads or threads())
    return cent, assign[:n], inertia.value, iters.value


# ---- product.rs ----
def pq_layout(dim: int, m: int):
    w = np.zeros(m, dtype=np.uint32)
    o = np.zeros(m + 1, dtype=np.uint32)
    lib().pxo_pq_layout(dim, m, _p(w), _p(o))
    return w, o


def pq_train(training, m: int, max_iterations: int = 25, seed: int = 0x5EED1EAF, nthreads=None):
    t = f32a(training)
    n, dim = t.shape
    books = np.zeros(256 * dim, dtype=np.float32)
    inertia = C.c_double()
    iters = C.c_uint64()
    rc = lib().pxo_pq_train(_p(t), n, dim, m, max_iterations, seed, _p(books), C.byref(inertia),
                            C.byref(iters), nthreads or threads())
    if rc != 0:
        raise ValueError("invalid PQ configuration")
    return books, inertia.value, iters.value


def pq_encode(books, dim: int, m: int, vectors) -> np.ndarray:
    v = f32a(vectors).reshape(-1, dim)
    out = np.zeros((v.shape[0], m), dtype=np.uint8)
    lib().pxo_pq_encode(_p(f32a(books)), dim, m, _p(v), v.shape[0], _p(out))
    return out


def pq_decode(books, dim: int, m: int, codes) -> np.ndarray:
    c = np.ascontiguousarray(codes, dtype=np.uint8).reshape(-1, m)
    out = np.zeros((c.shape[0], dim), dtype=np.float32)
    lib().pxo_pq_decode(_p(f32a(books)), dim, m, _p(c), c.shape[0], _p(out))
    return out


def pq_tables(books, dim: int, m: int, query):
    sq = np.zeros(m * 256, dtype=np.float32)
    dt = np.zeros(m * 256, dtype=np.float32)
    lib().pxo_pq_distance_table(_p(f32a(books)), dim, m, _p(f32a(query)), _p(sq), _p(dt))
    return sq, dt


def pq_adc_squared(table, m: int, code) -> float:
    c = np.ascontiguousarray(code, dtype=np.uint8)
    return lib().pxo_pq_adc_squared(_p(f32a(table)), m, _p(c))


# ---- scalar.rs ----
def sq_train(training, mode: int):
    t = f32a(training)
    n, dim = t.shape
    g = 1 if mode == RANGE_GLOBAL else dim
    mn, sc, inv = (np.zeros(g, dtype=np.float32) for _ in range(3))
    bad = lib().pxo_sq_train(_p(t), n, dim, mode, _p(mn), _p(sc), _p(inv))
    if bad >= 0:
        raise ValueError(f"non-finite component {bad}")
    return mn, sc, inv


def sq_encode(mn, inv, dim: int, mode: int, code_type: int, vectors) -> np.ndarray:
    v = f32a(vectors).reshape(-1, dim)
    out = np.zeros((v.shape[0], dim), dtype=np.uint8)
    lib().pxo_sq_encode(_p(mn), _p(inv), dim, mode, code_type, _p(v), v.shape[0], _p(out))
    return out


def sq_decode(mn, sc, dim: int, mode: int, code_type: int, codes) -> np.ndarray:
    c = np.ascontiguousarray(codes, dtype=np.uint8).reshape(-1, dim)
    out = np.zeros((c.shape[0], dim), dtype=np.float32)
    lib().pxo_sq_decode(_p(mn), _p(sc), dim, mode, code_type, _p(c), c.shape[0], _p(out))
    return out


def sq_asym_l2(mn, sc, dim: int, mode: int, code_type: int, query, code) -> float:
    c = np.ascontiguousarray(code, dtype=np.uint8)
    return lib().pxo_sq_asymmetric_squared_l2(_p(mn), _p(sc), dim, mode, code_type, _p(f32a(query)), _p(c))


# ---- ivfpq.rs ----
def sq_query_s8(scale, dim: int, mode: int, query) -> np.ndarray:
    """The query in code space as s8 (the SQ search's step 1)."""
    sc = f32a(scale)
    q = f32a(query)
    out = np.zeros(dim, np.int8)
    lib().pxo_sq_query_s8(_p(sc), dim, mode, _p(q), _p(out))
    return out


def sq_search(scale, mode: int, codes, rows, queries, k: int, overfetch: int, metric: int,
              ids=None, accepted=None, nthreads=None):
    """Over-fetch on s8 scores, exact re-rank to k. ``codes`` (n, dim) I8 codes
    and ``rows`` (n, dim) prepared vectors in rank order; ``ids`` the VectorId of
    each rank (ascending), ``accepted`` one byte per rank or None."""
    c = np.ascontiguousarray(codes).view(np.int8)
    r = f32a(rows).reshape(c.shape)
    n, dim = c.shape
    q = f32a(queries).reshape(-1, dim)
    nq = q.shape[0]
    oid = np.zeros((nq, max(k, 1)), np.uint64)
    od = np.zeros((nq, max(k, 1)), np.float32)
    ol = np.zeros(nq, np.uint32)
    idv = None if ids is None else np.ascontiguousarray(ids, np.uint64)
    acc = None if accepted is None else np.ascontiguousarray(accepted, np.uint8)
    lib().pxo_sq_search(_p(f32a(scale)), dim, mode, _p(c), _p(r), _p(idv), _p(acc), n, metric, _p(q), nq,
                        k, overfetch, _p(oid), _p(od), _p(ol), nthreads or threads())
    return oid[:, :k], od[:, :k], ol


def ivfpq_train(vectors, nlist: int, m: int, max_iterations: int = 25, training_sample: int = 100_000,
                seed: int = 0x1FF9C0D, live=None, coarse_init=None, pq_init=None, nthreads=None):
    v = f32a(vectors)
    n, dim = v.shape
    cent = np.zeros((nlist, dim), dtype=np.float32)
    books = np.zeros(256 * dim, dtype=np.float32)
    list_of = np.zeros(n, dtype=np.uint32)
    codes = np.zeros((n, m), dtype=np.uint8)
    rep = IvfReport()
    live = None if live is None else np.ascontiguousarray(live, dtype=np.uint8)
    ci = None if coarse_init is None else f32a(coarse_init)
    pi = None if pq_init is None else f32a(pq_init)
    produced = lib().pxo_ivfpq_train(_p(v), _p(live), n, dim, nlist, m, max_iterations, training_sample,
                                     seed, _p(ci), _p(pi), _p(cent), _p(books), _p(list_of), _p(codes),
                                     C.byref(rep), nthreads or threads())
    return cent[:produced], books, list_of, codes, rep


def ivfpq_search(vectors, centroids, books, m: int, list_of, codes, queries, k: int, nprobe: int,
                 rerank: int = 0, metric: int = EUCLIDEAN, ids=None, live=None, bitmap=None, nthreads=None):
    v = None if vectors is None else f32a(vectors)
    q = f32a(queries)
    nq, dim = q.shape
    nslots = len(list_of)
    cent = f32a(centroids)
    kk = max(k, 1)
    out_ids = np.zeros((nq, kk), dtype=np.uint64)
    out_d = np.zeros((nq, kk), dtype=np.float32)
    out_len = np.zeros(nq, dtype=np.uint32)
    lo = np.ascontiguousarray(list_of, dtype=np.uint32)
    cd = np.ascontiguousarray(codes, dtype=np.uint8)
    ids = None if ids is None else np.ascontiguousarray(ids, dtype=np.uint64)
    live = None if live is None else np.ascontiguousarray(live, dtype=np.uint8)
    bitmap = None if bitmap is None else np.ascontiguousarray(bitmap, dtype=np.uint64)
    lib().pxo_ivfpq_search(_p(v), _p(ids), _p(live), nslots, dim, metric, _p(cent), cent.shape[0],
                           _p(f32a(books)), m, _p(lo), _p(cd), _p(q), nq, k, nprobe, rerank, _p(bitmap),
                           _p(out_ids), _p(out_d), _p(out_len), nthreads or threads())
    return out_ids[:, :k], out_d[:, :k], out_len


def ivfpq_search_csr(vectors, centroids, books, m: int, list_off, list_slot, codes, queries, k: int, nprobe: int,
                     rerank: int = 0, metric: int = EUCLIDEAN, nthreads=None):
    """ivfpq_search over prebuilt lists (CSR), slots as ids, all live."""
    v = None if vectors is None else f32a(vectors)
    q = f32a(queries)
    nq, dim = q.shape
    cent = f32a(centroids)
    kk = max(k, 1)
    out_ids = np.zeros((nq, kk), dtype=np.uint64)
    out_d = np.zeros((nq, kk), dtype=np.float32)
    out_len = np.zeros(nq, dtype=np.uint32)
    lo = np.ascontiguousarray(list_off, dtype=np.uint32)
    ls = np.ascontiguousarray(list_slot, dtype=np.uint32)
    cd = np.ascontiguousarray(codes, dtype=np.uint8)
    lib().pxo_ivfpq_search_csr(_p(v), None, None, len(cd), dim, metric, _p(cent), cent.shape[0], _p(f32a(books)), m,
                               _p(lo), _p(ls), _p(cd), _p(q), nq, k, nprobe, rerank, None, _p(out_ids), _p(out_d),
                               _p(out_len), nthreads or threads())
    return out_ids[:, :k], out_d[:, :k], out_len


# ---- crates/proxima-server/src/filter.rs (the checker for the device filter) ----
def _filter_scalar(v):
    """scalar_value (filter.rs:171-183): (variant, payload)."""
    if isinstance(v, bool):
        return ("Bool", v)
    if isinstance(v, str):
        return ("Text", v)
    if isinstance(v, (int, float, np.integer, np.floating)):
        f = float(v)
        if f == f and abs(f) != float("inf") and f == int(f) and abs(f) < 9.007e15:
            return ("Int", int(f))
        return ("Float", f)
    raise ValueError("filter needs a string, number or boolean")


def _meta_value(v):
    """MetadataValue of a Python value (crates/proxima-core/src/metadata.rs:21-31), no coercion."""
    if v is None:
        return None
    if isinstance(v, bool):
        return ("Bool", v)
    if isinstance(v, (int, np.integer)):
        return ("Int", int(v))
    if isinstance(v, (float, np.floating)):
        return ("Float", float(v))
    return ("Text", v)


def _f64_total_key(f):
    import struct
    b = struct.unpack("<q", struct.pack("<d", f))[0]
    return b ^ ((b >> 63) & 0x7FFFFFFFFFFFFFFF)


def _number_compare(bound, value):
    """Number::compare (filter.rs:81-97)."""
    if bound[0] == "Int" and value[0] == "Int":
        return (value[1] > bound[1]) - (value[1] < bound[1])
    if value[0] == "Float" and bound[0] in ("Float", "Int"):
        a, b = _f64_total_key(value[1]), _f64_total_key(float(bound[1]))
        return (a > b) - (a < b)
    return None


def metadata_filter_accepts(filter_obj: dict, metadata: dict) -> bool:
    """MetadataFilter::parse (filter.rs:122-200) then Filter::accepts (:216-256), restated."""
    conds = []
    for field, cond in filter_obj.items():
        if isinstance(cond, dict):
            for op, operand in cond.items():
                if op == "in":
                    conds.append((field, op, [_filter_scalar(x) for x in operand]))
                elif op == "exists":
                    conds.append((field, op, bool(operand)))
                elif op in ("gt", "gte", "lt", "lte"):
                    conds.append((field, op, _filter_scalar(operand)))
                else:
                    conds.append((field, op, _filter_scalar(operand)))
        else:
            conds.append((field, "eq", _filter_scalar(cond)))
    conds.sort(key=lambda c: c[0])
    for field, op, operand in conds:
        value = _meta_value(metadata.get(field)) if metadata else None
        if op == "exists":
            held = (value is not None) == operand
        elif value is None:
            held = False
        elif op == "eq":
            held = value[0] == operand[0] and value[1] == operand[1]
        elif op == "ne":
            held = not (value[0] == operand[0] and value[1] == operand[1])
        elif op == "in":
            held = any(value[0] == o[0] and value[1] == o[1] for o in operand)
        else:
            o = _number_compare(operand, value)
            held = o is not None and {"gt": o == 1, "gte": o in (0, 1), "lt": o == -1, "lte": o in (-1, 0)}[op]
        if not held:
            return False
    return True


def slot_bitmap(accepted) -> np.ndarray:
    """Bitmap over slots from one bool per slot (bit s & 63 of word s / 64)."""
    a = np.asarray(accepted, dtype=bool)
    words = np.zeros((a.size + 63) // 64, dtype=np.uint64)
    if a.size:
        packed = np.packbits(a, bitorder="little")
        packed = np.concatenate([packed, np.zeros(words.size * 8 - packed.size, dtype=np.uint8)])
        words[:] = packed.view(np.uint64)
    return words


# ---------------------------------------------------------------------------
# Snapshot codec (crates/proxima-store/src/snapshot.rs, codec.rs, crc.rs)
# ---------------------------------------------------------------------------
import struct as _struct

SNAP_MAGIC = b"PROXSNAP"
_METRIC_TAG = {EUCLIDEAN: 1, COSINE: 2, INNER_PRODUCT: 3, MANHATTAN: 4}
_TAG_METRIC = {v: k for k, v in _METRIC_TAG.items()}


class SnapshotError(Exception):
    """kind "corrupt" (ProximaError::Corruption, with the structure) or "config"
    (ProximaError::Configuration, with the parameter)."""

    def __init__(self, kind, where, detail):
        super().__init__(f"{kind} {where}: {detail}")
        self.kind, self.where, self.detail = kind, where, detail


def crc32c(data, crc: int = 0) -> int:
    """crc32c_append (crc.rs:64-79), the oracle's byte-at-a-time restatement."""
    b = bytes(data)
    return int(lib().pxo_crc32c_append(crc, b, len(b)))


def encode_metadata_entry(m) -> bytes:
    """Writer::metadata (codec.rs:170-200): field count, then (key, tag, value) with keys in byte order."""
    m = m or {}
    out = [_struct.pack("<I", len(m))]
    for key in sorted(m, key=lambda k: k.encode("utf-8")):
        kb = key.encode("utf-8")
        out.append(_struct.pack("<I", len(kb)) + kb)
        v = m[key]
        if isinstance(v, bool):
            out.append(_struct.pack("<BB", 4, int(v)))
        elif isinstance(v, (int, np.integer)):
            out.append(_struct.pack("<BQ", 2, int(v) & 0xFFFFFFFFFFFFFFFF))
        elif isinstance(v, (float, np.floating)):
            out.append(_struct.pack("<Bd", 3, float(v)))
        else:
            tb = str(v).encode("utf-8")
            out.append(_struct.pack("<BI", 1, len(tb)) + tb)
    return b"".join(out)


def snapshot_encode_ivfpq(dim, metric, config, ids, metadata, vectors, codes, list_of, centroids, codebooks,
                          report=None) -> bytes:
    """encode (snapshot.rs:120-200, IVF-PQ arm) and the header (:190-199).
    `config` is a dict of IvfPqConfig's fields, `ids` a list of VectorId or None
    per slot, `metadata` a list of dicts, `report` a dict of TrainingReport's
    fields or None."""
    body = bytearray(_struct.pack("<IB", dim, _METRIC_TAG[metric]))
    body += bytes([3])
    c = config
    body += _struct.pack("<IIIIQIIQB", c["nlist"], c["subspaces"], c["nprobe"], c["rerank"], c["seed"],
                         c["max_iterations"], c["training_sample"], c["train_threshold"], int(bool(c["retain_vectors"])))
    body += _struct.pack("<I", len(ids))
    for i in ids:
        body += _struct.pack("<BQ", 0, 0) if i is None else _struct.pack("<BQ", 1, int(i))
    body += _struct.pack("<I", len(metadata))
    for m in metadata:
        body += encode_metadata_entry(m)
    for arr, dt in ((vectors, "<f4"), (codes, "u1"), (list_of, "<u4"), (centroids, "<f4"), (codebooks, "<f4")):
        a = np.ascontiguousarray(np.asarray(arr).reshape(-1), dtype=dt)
        body += _struct.pack("<I", a.size) + a.tobytes()
    if report is None:
        body += b"\0"
    else:
        r = report
        body += _struct.pack("<BIdIdII", 1, r["sampled"], r["coarse_inertia"], r["coarse_iterations"],
                             r["residual_inertia"], r["populated_lists"], r["largest_list"])
    head = SNAP_MAGIC + _struct.pack("<IIIQ", 1, 0x01020304, 0, len(body))
    return bytes(head) + bytes(body) + _struct.pack("<I", crc32c(body))


class _Reader:
    """codec.rs Reader (:207-392): bounded reads, length prefixes checked against what remains."""

    def __init__(self, b, structure):
        self.b, self.pos, self.structure = b, 0, structure

    def remaining(self):
        return len(self.b) - self.pos

    def take(self, n):
        if self.remaining() < n:
            raise SnapshotError("corrupt", self.structure,
                                f"truncated at byte {self.pos}: wanted {n} more, {self.remaining()} remain")
        out = self.b[self.pos:self.pos + n]
        self.pos += n
        return out

    def u8(self):
        return self.take(1)[0]

    def u32(self):
        return _struct.unpack("<I", self.take(4))[0]

    def u64(self):
        return _struct.unpack("<Q", self.take(8))[0]

    def f64(self):
        return _struct.unpack("<d", self.take(8))[0]

    def len_prefix(self, elem):
        n = self.u32()
        if n * max(elem, 1) > self.remaining():
            raise SnapshotError("corrupt", self.structure, f"length prefix at byte {self.pos - 4} claims {n} elements")
        return n

    def text(self):
        b = self.take(self.len_prefix(1))
        try:
            return bytes(b).decode("utf-8")
        except UnicodeDecodeError as e:
            raise SnapshotError("corrupt", self.structure, f"field is not UTF-8: {e}") from None

    def array(self, dt, elem):
        n = self.len_prefix(elem)
        return np.frombuffer(bytes(self.take(n * elem)), dtype=dt).copy()

    def metadata(self):
        m = {}
        for _ in range(self.len_prefix(4)):
            key = self.text()
            tag = self.u8()
            if tag == 1:
                m[key] = self.text()
            elif tag == 2:
                m[key] = _struct.unpack("<q", self.take(8))[0]
            elif tag == 3:
                m[key] = self.f64()
            elif tag == 4:
                m[key] = self.u8() != 0
            else:
                raise SnapshotError("corrupt", self.structure, f"metadata value tag {tag} is not one of 1..=4")
        return m


def snapshot_decode_ivfpq(image) -> dict:
    """decode (snapshot.rs:192-269) of an IVF-PQ snapshot with verify (:331-380)
    and IvfPqIndex::new / IvfPqConfig::validate / from_parts (ivfpq.rs:259-302,
    481-491, 624-717). Returns the parts as a dict; raises SnapshotError."""
    b = bytes(image)
    if len(b) < 32:
        raise SnapshotError("corrupt", "snapshot header", f"{len(b)} bytes is shorter than the header plus checksum")
    if b[:8] != SNAP_MAGIC:
        raise SnapshotError("corrupt", "snapshot header", "bad magic")
    version, order, reserved, body_len = _struct.unpack("<IIIQ", b[8:28])
    if version != 1:
        raise SnapshotError("corrupt", "snapshot header", f"format version {version}")
    if reserved != 0:
        raise SnapshotError("corrupt", "snapshot header", "reserved word is not zero")
    if order != 0x01020304:
        raise SnapshotError("corrupt", "snapshot header", "byte-order mark")
    if len(b) != 28 + body_len + 4:
        raise SnapshotError("corrupt", "snapshot", "header length disagrees with the file")
    body = b[28:28 + body_len]
    expected = _struct.unpack("<I", b[28 + body_len:])[0]
    if crc32c(body) != expected:
        raise SnapshotError("corrupt", "snapshot", "checksum mismatch")
    rd = _Reader(body, "snapshot body")
    dim = rd.u32()
    tag = rd.u8()
    if tag not in _TAG_METRIC:
        raise SnapshotError("corrupt", "snapshot body", f"metric tag {tag} is not one of 1..=4")
    metric = _TAG_METRIC[tag]
    if dim < 1 or dim > 1 << 20:
        raise SnapshotError("config", "dim", "out of range")
    kind = rd.u8()
    if kind not in (1, 2, 3):
        raise SnapshotError("corrupt", "snapshot body", f"index kind {kind} is not one of 1..=3")
    if kind != 3:
        return {"kind": kind, "dim": dim, "metric": metric}
    cfg = dict(zip(("nlist", "subspaces", "nprobe", "rerank"), (rd.u32(), rd.u32(), rd.u32(), rd.u32())))
    cfg["seed"] = rd.u64()
    cfg["max_iterations"], cfg["training_sample"] = rd.u32(), rd.u32()
    cfg["train_threshold"] = rd.u64()
    cfg["retain_vectors"] = rd.u8() != 0
    ids = []
    for _ in range(rd.len_prefix(9)):
        present = rd.u8() != 0
        raw = rd.u64()
        ids.append(raw if present else None)
    metadata = [rd.metadata() for _ in range(rd.len_prefix(4))]
    vectors = rd.array("<f4", 4)
    codes = rd.array("u1", 1)
    list_of = rd.array("<u4", 4)
    centroids = rd.array("<f4", 4)
    codebooks = rd.array("<f4", 4)
    report = None
    if rd.u8() != 0:
        report = {"sampled": rd.u32(), "coarse_inertia": rd.f64(), "coarse_iterations": rd.u32(),
                  "residual_inertia": rd.f64(), "populated_lists": rd.u32(), "largest_list": rd.u32()}
    # IvfPqIndex::new and IvfPqConfig::validate
    if metric not in (EUCLIDEAN, COSINE):
        raise SnapshotError("config", "metric", "IVF-PQ supports euclidean and cosine only")
    for name, bad in (("nlist", cfg["nlist"] == 0),
                      ("subspaces", cfg["subspaces"] == 0 or cfg["subspaces"] > dim),
                      ("nprobe", cfg["nprobe"] == 0 or cfg["nprobe"] > cfg["nlist"]),
                      ("max_iterations", cfg["max_iterations"] == 0),
                      ("training_sample", cfg["training_sample"] == 0),
                      ("rerank", cfg["rerank"] > 0 and not cfg["retain_vectors"])):
        if bad:
            raise SnapshotError("config", name, "rejected by IvfPqConfig::validate")
    # from_parts
    n, m = len(ids), cfg["subspaces"]
    if len(metadata) != n:
        raise SnapshotError("corrupt", "ivfpq index", "metadata count")
    if vectors.size and vectors.size != n * dim:
        raise SnapshotError("corrupt", "ivfpq index", "vectors length")
    if codes.size and (codes.size != n * m or list_of.size != n):
        raise SnapshotError("corrupt", "ivfpq index", "codes or list assignments length")
    lists = cfg["nlist"]
    if centroids.size:
        if centroids.size % dim:
            raise SnapshotError("corrupt", "ivfpq centroids", "not a multiple of the dimension")
        if codebooks.size != 256 * dim:
            raise SnapshotError("corrupt", "product quantizer", "codebook length")
        lists = centroids.size // dim
    seen = {}
    for slot, i in enumerate(ids):
        if i is not None:
            if i in seen:
                raise SnapshotError("corrupt", "ivfpq index", f"id {i} appears at two slots")
            seen[i] = slot
    for slot, lst in enumerate(list_of.tolist()):
        if lst == 0xFFFFFFFF or ids[slot] is None:
            continue
        if lst >= lists:
            raise SnapshotError("corrupt", "ivfpq index", f"slot {slot} names list {lst} of {lists}")
    if rd.remaining():
        raise SnapshotError("corrupt", "snapshot body", f"{rd.remaining()} trailing bytes after the final field")
    return {"kind": 3, "dim": dim, "metric": metric, "config": cfg, "ids": ids, "metadata": metadata,
            "vectors": vectors, "codes": codes, "list_of": list_of, "centroids": centroids, "codebooks": codebooks,
            "report": report, "lists": lists}


def snapshot_encode_flat(dim, metric, ids, data, metadata) -> bytes:
    """encode (snapshot.rs:124-130) of a flat index: the store as encode_store (:383-405) writes it."""
    body = bytearray(_struct.pack("<IB", dim, _METRIC_TAG[metric])) + bytes([1])
    body += _struct.pack("<I", len(ids))
    for i in ids:
        body += _struct.pack("<BQ", 0, 0) if i is None else _struct.pack("<BQ", 1, int(i))
    a = np.ascontiguousarray(np.asarray(data).reshape(-1), dtype="<f4")
    body += _struct.pack("<I", a.size) + a.tobytes()
    body += _struct.pack("<I", len(metadata))
    for m in metadata:
        body += encode_metadata_entry(m)
    head = SNAP_MAGIC + _struct.pack("<IIIQ", 1, 0x01020304, 0, len(body))
    return bytes(head) + bytes(body) + _struct.pack("<I", crc32c(body))
