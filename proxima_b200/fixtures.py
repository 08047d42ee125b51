"""Synthetic workloads (ctypes over ``lib/libpxfix.so``; see csrc/fixtures.cpp).

Seeds are fixed choices of this build; the configurations mirror the
benchmark shapes (quickstart C1, integer blobs C2/C4, unit-sphere blobs C3/C5).
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

_LIB = Path(__file__).resolve().parent / "lib" / "libpxfix.so"
_lib = None

C2_CENTRES, C2_BASE, C2_QUERIES = 0xC2C20001, 0xC2C20011, 0xC2C20002
C3_CENTRES, C3_POINTS = 0xC3C30001, 0xC3C30011
C4_CENTRES, C4_BASE, C4_QUERIES = 0xC4C40001, 0xC4C40011, 0xC4C40002
C5_CENTRES, C5_BASE, C5_QUERIES, C5_YEARS = 0xC5C50001, 0xC5C50011, 0xC5C50002, 0xC5C50003


def _load():
    global _lib
    if _lib is None:
        if not _LIB.exists():
            raise RuntimeError(f"{_LIB} is missing: run `python -m proxima_b200.build`")
        lib = C.CDLL(str(_LIB))
        vp, u64, f64, i32 = C.c_void_p, C.c_uint64, C.c_double, C.c_int
        lib.pxf_quickstart.argtypes = [u64, u64, vp]
        lib.pxf_splitmix_corpus.argtypes = [u64, u64, u64, vp]
        lib.pxf_blobs_u8.argtypes = [u64, u64, u64, u64, u64, u64, f64, vp, i32]
        lib.pxf_blobs_f32.argtypes = [u64, u64, u64, u64, u64, u64, f64, vp, i32]
        lib.pxf_blobs_u8_strided.argtypes = [u64, u64, u64, u64, u64, u64, u64, f64, vp, i32]
        lib.pxf_sphere_blobs.argtypes = [u64, u64, u64, u64, u64, u64, f64, vp, i32]
        lib.pxf_uniform_int.argtypes = [u64, u64, u64, C.c_int64, u64, vp]
        for f in (lib.pxf_quickstart, lib.pxf_splitmix_corpus, lib.pxf_blobs_u8, lib.pxf_blobs_f32,
                  lib.pxf_blobs_u8_strided,
                  lib.pxf_sphere_blobs, lib.pxf_uniform_int):
            f.restype = None
        _lib = lib
    return _lib


def _threads() -> int:
    return max(1, min(32, os.cpu_count() or 1))


def quickstart(count: int = 5000, dim: int = 64) -> np.ndarray:
    """examples/quickstart.rs:25-36 (config C1)."""
    out = np.empty((count, dim), dtype=np.float32)
    _load().pxf_quickstart(count, dim, out.ctypes.data)
    return out


def splitmix_corpus(count: int, seed: int, dim: int = 128) -> np.ndarray:
    """crates/proxima-quantize/tests/recall.rs:57-98."""
    out = np.empty((count, dim), dtype=np.float32)
    _load().pxf_splitmix_corpus(count, dim, seed, out.ctypes.data)
    return out


def blobs_u8(n: int, dim: int, nblobs: int, centre_seed: int, noise_seed: int,
             sigma: float = 20.0, row_begin: int = 0) -> np.ndarray:
    """Integer Gaussian blobs in [0,255]^dim stored as f32 (configs C2, C4)."""
    out = np.empty((n, dim), dtype=np.float32)
    _load().pxf_blobs_u8(row_begin, n, dim, nblobs, centre_seed, noise_seed, sigma,
                         out.ctypes.data, _threads())
    return out


def blobs_u8_strided(n: int, stride: int, dim: int, nblobs: int, centre_seed: int, noise_seed: int,
                     sigma: float = 20.0, row_first: int = 0) -> np.ndarray:
    """Rows row_first + i * stride (i < n) of blobs_u8's stream: a stride sample."""
    out = np.empty((n, dim), dtype=np.float32)
    _load().pxf_blobs_u8_strided(row_first, stride, n, dim, nblobs, centre_seed, noise_seed, sigma,
                                 out.ctypes.data, _threads())
    return out


def blobs_f32(n: int, dim: int, nblobs: int, centre_seed: int, noise_seed: int,
              sigma: float = 20.0, row_begin: int = 0) -> np.ndarray:
    """The C2 blobs without rounding or clipping: real-valued rows."""
    out = np.empty((n, dim), dtype=np.float32)
    _load().pxf_blobs_f32(row_begin, n, dim, nblobs, centre_seed, noise_seed, sigma,
                          out.ctypes.data, _threads())
    return out


def sphere_blobs(n: int, dim: int, nblobs: int, centre_seed: int, noise_seed: int,
                 sigma: float, row_begin: int = 0) -> np.ndarray:
    """L2-normalised blobs around unit-sphere centres (configs C3, C5)."""
    out = np.empty((n, dim), dtype=np.float32)
    _load().pxf_sphere_blobs(row_begin, n, dim, nblobs, centre_seed, noise_seed, sigma,
                             out.ctypes.data, _threads())
    return out


def uniform_int(n: int, seed: int, lo: int, span: int, row_begin: int = 0) -> np.ndarray:
    out = np.empty(n, dtype=np.int64)
    _load().pxf_uniform_int(row_begin, n, seed, lo, span, out.ctypes.data)
    return out


def c2_database(n: int = 1_000_000, dim: int = 128) -> np.ndarray:
    return blobs_u8(n, dim, 1024, C2_CENTRES, C2_BASE, 20.0)


def c2_queries(nq: int = 10_000, dim: int = 128) -> np.ndarray:
    return blobs_u8(nq, dim, 1024, C2_CENTRES, C2_QUERIES, 20.0)


C3_INIT = 0xC3C30003


def c3_points(n: int = 1_000_000, dim: int = 96, nblobs: int = 4096) -> np.ndarray:
    """Config C3: normalise(centre + N(0, 0.05^2)) around 4,096 unit-sphere centres."""
    return sphere_blobs(n, dim, nblobs, C3_CENTRES, C3_POINTS, 0.05)


def sample_rows(n: int, k: int, seed: int) -> np.ndarray:
    """k distinct row indices of [0, n): the k smallest splitmix64(seed, i) keys
    (ties by index), in ascending key order. The seeded random-sample init of C3."""
    i = np.arange(n, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = (np.uint64(seed) + (i + np.uint64(1)) * np.uint64(0x9E3779B97F4A7C15))
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z = z ^ (z >> np.uint64(31))
    order = np.lexsort((i, z))
    return order[:k].astype(np.int64)


def c3_init(points: np.ndarray, k: int = 4096, seed: int = C3_INIT) -> np.ndarray:
    return np.ascontiguousarray(points[sample_rows(len(points), k, seed)])
