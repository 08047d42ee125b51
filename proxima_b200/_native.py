"""ctypes bindings for ``libproxima_cuda.so`` (the C ABI in ``include/proxima_cuda.h``).

The library is built in-tree by ``proxima_b200.build``. There is no fallback:
if the library is missing or no B200 is visible, every call fails loudly.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

from .errors import raise_for_status

LIB_DIR = Path(__file__).resolve().parent / "lib"
# PXC_LIBRARY selects another build of the same ABI (e.g. a packaged copy).
LIB_PATH = Path(os.environ.get("PXC_LIBRARY", str(LIB_DIR / "libproxima_cuda.so")))

u8p = C.POINTER(C.c_uint8)
u32p = C.POINTER(C.c_uint32)
u64p = C.POINTER(C.c_uint64)
f32p = C.POINTER(C.c_float)
f64p = C.POINTER(C.c_double)
vp = C.c_void_p


class PxcError(C.Structure):
    _fields_ = [
        ("code", C.c_int32),
        ("a", C.c_uint64),
        ("b", C.c_uint64),
        ("parameter", C.c_char * 32),
        ("detail", C.c_char * 256),
    ]


class PxcKmeansInfo(C.Structure):
    _fields_ = [
        ("k", C.c_uint32),
        ("iterations", C.c_uint32),
        ("inertia", C.c_double),
        ("path", C.c_uint32),
        ("reseeded", C.c_uint32),
        ("rescanned", C.c_uint64),
        ("screen_passes", C.c_uint32),
        ("screen_ms", C.c_float),
    ]


class PxcIvfpqReport(C.Structure):
    _fields_ = [
        ("sampled", C.c_uint64),
        ("coarse_inertia", C.c_double),
        ("coarse_iterations", C.c_uint64),
        ("residual_inertia", C.c_double),
        ("populated_lists", C.c_uint64),
        ("largest_list", C.c_uint64),
        ("produced", C.c_uint64),
        ("pq_iterations", C.c_uint64),
    ]


class PxcIvfpqConfig(C.Structure):
    _fields_ = [
        ("nlist", C.c_uint32),
        ("subspaces", C.c_uint32),
        ("nprobe", C.c_uint32),
        ("rerank", C.c_uint32),
        ("seed", C.c_uint64),
        ("max_iterations", C.c_uint32),
        ("training_sample", C.c_uint32),
        ("train_threshold", C.c_uint64),
        ("retain_vectors", C.c_uint32),
        ("reserved", C.c_uint32),
    ]


class PxcSnapshotInfo(C.Structure):
    _fields_ = [
        ("format_version", C.c_uint32),
        ("kind", C.c_uint32),
        ("dim", C.c_uint32),
        ("metric", C.c_int32),
        ("body_bytes", C.c_uint64),
        ("nslots", C.c_uint64),
        ("live", C.c_uint64),
        ("metadata_offset", C.c_uint64),
        ("metadata_bytes", C.c_uint64),
        ("config", PxcIvfpqConfig),
        ("trained", C.c_uint32),
        ("lists", C.c_uint32),
        ("has_vectors", C.c_uint32),
        ("has_report", C.c_uint32),
        ("report", PxcIvfpqReport),
    ]


class PxcRng(C.Structure):
    """pxc_rng: a ChaCha8Rng as rand_chacha exposes it (seed, stream, word position)."""

    _fields_ = [
        ("seed", C.c_uint8 * 32),
        ("stream", C.c_uint64),
        ("word_pos_lo", C.c_uint64),
        ("word_pos_hi", C.c_uint64),
    ]


class PxcCondition(C.Structure):
    """pxc_condition: one compiled MetadataFilter condition on one device column."""

    _fields_ = [("column", C.c_uint32), ("op", C.c_uint32), ("tag", C.c_uint32), ("count", C.c_uint32),
                ("value", C.c_int64)]


class PxcOperand(C.Structure):
    _fields_ = [("tag", C.c_uint32), ("reserved", C.c_uint32), ("value", C.c_int64)]


class PxcIntRange(C.Structure):
    """pxc_int_range: lo <= value <= hi on an integer metadata column."""

    _fields_ = [
        ("column", C.c_uint32),
        ("reserved", C.c_uint32),
        ("lo", C.c_int64),
        ("hi", C.c_int64),
    ]


# name -> (restype, argtypes); every symbol include/proxima_cuda.h declares.
SIGNATURES: dict[str, tuple] = {
    "pxc_abi_version": (C.c_uint32, []),
    "pxc_ctx_create": (C.c_int32, [C.POINTER(C.c_int), C.c_int, C.POINTER(vp), C.POINTER(PxcError)]),
    "pxc_ctx_destroy": (None, [vp]),
    "pxc_ctx_set_wait_limit": (C.c_int32, [vp, C.c_uint32, C.POINTER(PxcError)]),
    "pxc_flat_create": (C.c_int32, [vp, C.c_uint32, C.c_int32, C.POINTER(vp), C.POINTER(PxcError)]),
    "pxc_flat_destroy": (None, [vp]),
    "pxc_flat_sync": (C.c_int32, [vp, vp, vp, vp, C.c_uint64, C.c_uint64, C.POINTER(PxcError)]),
    "pxc_flat_truncate": (C.c_int32, [vp, C.c_uint64, C.POINTER(PxcError)]),
    "pxc_flat_len": (C.c_uint64, [vp]),
    "pxc_flat_search": (C.c_int32, [vp, vp, C.c_uint32, C.c_uint32, vp, vp, vp, vp, C.POINTER(PxcError)]),
    "pxc_flat_search_device": (C.c_int32, [vp, vp, C.c_uint32, C.c_uint32, vp, vp, vp, vp, vp,
                                           C.POINTER(PxcError)]),
    "pxc_flat_path": (C.c_int32, [vp]),
    "pxc_flat_search_noalloc": (C.c_int32, [vp, vp, C.c_uint32, C.c_uint32, vp, vp, vp, vp,
                                            C.POINTER(PxcError)]),
    "pxc_flat_last_scan_ms": (C.c_float, [vp]),
    "pxc_flat_last_redone": (C.c_uint32, [vp]),
    "pxc_ctx_launch_count": (C.c_uint64, [vp]),
    "pxc_ctx_set_profiling": (C.c_int32, [vp, C.c_int32, C.POINTER(PxcError)]),
    "pxc_topk_merge": (C.c_int32, [vp, vp, vp, vp, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32,
                                   vp, vp, vp, vp, C.POINTER(PxcError)]),
    "pxc_ctx_set_option": (C.c_int32, [vp, C.c_char_p, C.c_int64, C.POINTER(PxcError)]),
    "pxc_columns_create": (C.c_int32, [vp, C.POINTER(vp), C.POINTER(PxcError)]),
    "pxc_columns_destroy": (None, [vp]),
    "pxc_columns_set": (C.c_int32, [vp, C.c_uint32, vp, vp, C.c_uint64, C.c_uint64, C.POINTER(PxcError)]),
    "pxc_columns_truncate": (C.c_int32, [vp, C.c_uint64, C.POINTER(PxcError)]),
    "pxc_columns_eval": (C.c_int32, [vp, C.c_uint64, vp, C.c_uint32, vp, C.c_uint32, vp, vp, C.POINTER(PxcError)]),
    "pxc_flat_search_where": (C.c_int32, [vp, vp, vp, C.c_uint32, vp, C.c_uint32, vp, C.c_uint32, C.c_uint32, vp, vp,
                                          vp, C.POINTER(PxcError)]),
    "pxc_ivfpq_search_where": (C.c_int32, [vp, vp, vp, C.c_uint32, vp, C.c_uint32, vp, C.c_uint32, C.c_uint32,
                                           C.c_uint32, C.c_uint32, vp, vp, vp, C.POINTER(PxcError)]),
    "pxc_comm_unique_id": (C.c_int32, [vp, C.POINTER(PxcError)]),
    "pxc_ctx_init_comm": (C.c_int32, [vp, vp, C.c_int32, C.c_int32, C.c_uint32, C.POINTER(PxcError)]),
    "pxc_ctx_comm_size": (C.c_int32, [vp]),
    "pxc_ctx_comm_rank": (C.c_int32, [vp]),
    "pxc_flat_search_sharded": (C.c_int32, [vp, vp, C.c_uint32, C.c_uint32, vp, vp, vp, vp, vp,
                                            C.POINTER(PxcError)]),
    "pxc_topk_exchange": (C.c_int32, [vp, vp, vp, vp, C.c_uint32, C.c_uint32, C.c_uint32, vp, vp, vp, vp,
                                      C.POINTER(PxcError)]),
    "pxc_rng_seed_from_u64": (C.c_int32, [C.c_uint64, C.POINTER(PxcRng), C.POINTER(PxcError)]),
    "pxc_rng_next_u32": (C.c_int32, [C.POINTER(PxcRng), vp, C.c_uint64, C.POINTER(PxcError)]),
    "pxc_rng_gen_index": (C.c_int32, [C.POINTER(PxcRng), C.c_uint64, C.POINTER(C.c_uint64), C.POINTER(PxcError)]),
    "pxc_rng_gen_f64": (C.c_int32, [C.POINTER(PxcRng), C.c_double, C.c_double, C.POINTER(C.c_double),
                                    C.POINTER(PxcError)]),
    "pxc_chacha_block": (C.c_int32, [vp, C.c_uint64, C.c_uint64, C.c_uint32, vp, C.POINTER(PxcError)]),
    "pxc_kmeans": (C.c_int32, [vp, vp, C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32, vp, C.POINTER(PxcRng),
                               vp, vp, C.POINTER(PxcKmeansInfo), C.POINTER(PxcError)]),
    "pxc_kmeans_device": (C.c_int32, [vp, vp, C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32, vp,
                                      C.POINTER(PxcRng), vp, vp, C.POINTER(PxcKmeansInfo), vp,
                                      C.POINTER(PxcError)]),
    "pxc_kmeans_sharded": (C.c_int32, [vp, vp, C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32, vp, vp, vp,
                                       C.POINTER(PxcKmeansInfo), vp, C.POINTER(PxcError)]),
    "pxc_pq_train": (C.c_int32, [vp, vp, C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint64, vp,
                                 C.POINTER(C.c_double), C.POINTER(C.c_uint64), C.POINTER(PxcError)]),
    "pxc_pq_train_device": (C.c_int32, [vp, vp, C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint64, vp,
                                        C.POINTER(C.c_double), C.POINTER(C.c_uint64), vp, C.POINTER(PxcError)]),
    "pxc_pq_encode": (C.c_int32, [vp, vp, C.c_uint32, C.c_uint32, vp, C.c_uint64, vp, C.POINTER(PxcError)]),
    "pxc_pq_encode_device": (C.c_int32, [vp, vp, C.c_uint32, C.c_uint32, vp, C.c_uint64, vp, vp,
                                         C.POINTER(PxcError)]),
    "pxc_pq_decode": (C.c_int32, [vp, vp, C.c_uint32, C.c_uint32, vp, C.c_uint64, vp, C.POINTER(PxcError)]),
    "pxc_pq_tables": (C.c_int32, [vp, vp, C.c_uint32, C.c_uint32, vp, C.c_uint32, vp, vp, C.POINTER(PxcError)]),
    "pxc_pq_tables_device": (C.c_int32, [vp, vp, C.c_uint32, C.c_uint32, vp, C.c_uint32, vp, vp, vp,
                                         C.POINTER(PxcError)]),
    "pxc_sq_asymmetric": (C.c_int32, [vp, vp, vp, C.c_uint32, C.c_int32, C.c_int32, C.c_int32, vp, C.c_uint32,
                                      vp, C.c_uint64, vp, C.POINTER(PxcError)]),
    "pxc_sq_asymmetric_device": (C.c_int32, [vp, vp, vp, C.c_uint32, C.c_int32, C.c_int32, C.c_int32, vp,
                                             C.c_uint32, vp, C.c_uint64, vp, vp, C.POINTER(PxcError)]),
    "pxc_ivfpq_create": (C.c_int32, [vp, C.c_uint32, C.c_int32, C.c_uint32, C.c_uint32, C.POINTER(vp),
                                     C.POINTER(PxcError)]),
    "pxc_ivfpq_destroy": (None, [vp]),
    "pxc_ivfpq_set_parts": (C.c_int32, [vp, vp, vp, C.POINTER(PxcError)]),
    "pxc_ivfpq_set_store": (C.c_int32, [vp, vp, vp, vp, C.c_uint64, C.POINTER(PxcError)]),
    "pxc_ivfpq_set_store_device": (C.c_int32, [vp, vp, vp, vp, C.c_uint64, C.POINTER(PxcError)]),
    "pxc_ivfpq_last_scan_ms": (C.c_float, [vp]),
    "pxc_ivfpq_last_scanned": (C.c_uint64, [vp]),
    "pxc_ivfpq_set_codes": (C.c_int32, [vp, vp, vp, C.POINTER(PxcError)]),
    "pxc_ivfpq_encode_all": (C.c_int32, [vp, C.POINTER(PxcError)]),
    "pxc_ivfpq_train": (C.c_int32, [vp, C.c_uint64, C.c_uint32, C.c_uint64, C.POINTER(PxcIvfpqReport),
                                    C.POINTER(PxcError)]),
    "pxc_ivfpq_get_parts": (C.c_int32, [vp, vp, vp, vp, vp, C.POINTER(C.c_uint32), C.POINTER(PxcError)]),
    "pxc_ivfpq_search": (C.c_int32, [vp, vp, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, vp, vp, vp, vp,
                                     C.POINTER(PxcError)]),
    "pxc_flat_search_sharded_owned": (C.c_int32, [vp, vp, C.c_uint32, C.c_uint32, vp, vp, vp, vp, vp,
                                                  C.POINTER(PxcError)]),
    "pxc_ctx_owned_range": (None, [vp, C.c_uint32, C.POINTER(C.c_uint32), C.POINTER(C.c_uint32)]),
    "pxc_ivfpq_search_sharded": (C.c_int32, [vp, vp, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, vp, vp,
                                             vp, vp, vp, C.POINTER(PxcError)]),
    "pxc_ivfpq_search_device": (C.c_int32, [vp, vp, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, vp, vp,
                                            vp, vp, vp, C.POINTER(PxcError)]),
    "pxc_crc32c_append": (C.c_uint32, [C.c_uint32, vp, C.c_uint64]),
    "pxc_crc32c_combine": (C.c_uint32, [C.c_uint32, C.c_uint32, C.c_uint64]),
    "pxc_crc32c_device": (C.c_int32, [vp, vp, C.c_uint64, C.POINTER(C.c_uint32), vp, C.POINTER(PxcError)]),
    "pxc_snapshot_peek": (C.c_int32, [vp, C.c_uint64, C.POINTER(PxcSnapshotInfo), C.POINTER(PxcError)]),
    "pxc_ivfpq_snapshot_load": (C.c_int32, [vp, vp, C.c_uint64, C.POINTER(vp), C.POINTER(PxcSnapshotInfo),
                                            C.POINTER(PxcError)]),
    "pxc_ivfpq_snapshot_save": (C.c_int32, [vp, C.POINTER(PxcIvfpqConfig), C.POINTER(PxcIvfpqReport), vp,
                                            C.c_uint64, vp, C.c_uint64, C.POINTER(C.c_uint64),
                                            C.POINTER(PxcError)]),
    "pxc_sq_train": (C.c_int32, [vp, vp, C.c_uint64, C.c_uint32, C.c_int32, vp, vp, vp, C.POINTER(PxcError)]),
    "pxc_sq_train_device": (C.c_int32, [vp, vp, C.c_uint64, C.c_uint32, C.c_int32, vp, vp, vp, vp,
                                        C.POINTER(PxcError)]),
    "pxc_sq_ranges_device": (C.c_int32, [vp, vp, C.c_uint64, C.c_uint32, C.c_int32, vp, vp, vp,
                                         C.POINTER(PxcError)]),
    "pxc_sq_encode": (C.c_int32, [vp, vp, vp, C.c_uint32, C.c_int32, C.c_int32, vp, C.c_uint64, vp,
                                  C.POINTER(PxcError)]),
    "pxc_sq_encode_device": (C.c_int32, [vp, vp, vp, C.c_uint32, C.c_int32, C.c_int32, vp, C.c_uint64, vp, vp,
                                         C.POINTER(PxcError)]),
    "pxc_sq_decode": (C.c_int32, [vp, vp, vp, C.c_uint32, C.c_int32, C.c_int32, vp, C.c_uint64, vp,
                                  C.POINTER(PxcError)]),
    "pxc_sq_create": (C.c_int32, [vp, C.c_uint32, C.c_int32, C.POINTER(vp), C.POINTER(PxcError)]),
    "pxc_sq_destroy": (None, [vp]),
    "pxc_sq_set_quantizer": (C.c_int32, [vp, C.c_int32, vp, vp, vp, C.POINTER(PxcError)]),
    "pxc_sq_get_quantizer": (C.c_int32, [vp, C.POINTER(C.c_int32), vp, vp, vp, C.POINTER(PxcError)]),
    "pxc_sq_train_store": (C.c_int32, [vp, C.c_int32, C.POINTER(PxcError)]),
    "pxc_sq_set_store": (C.c_int32, [vp, vp, vp, vp, C.c_uint64, C.POINTER(PxcError)]),
    "pxc_sq_set_store_device": (C.c_int32, [vp, vp, vp, vp, C.c_uint64, C.POINTER(PxcError)]),
    "pxc_sq_set_column": (C.c_int32, [vp, C.c_uint32, vp, vp, C.POINTER(PxcError)]),
    "pxc_sq_len": (C.c_uint64, [vp]),
    "pxc_sq_get_codes": (C.c_int32, [vp, vp, C.POINTER(PxcError)]),
    "pxc_sq_search": (C.c_int32, [vp, vp, C.c_uint32, C.c_uint32, C.c_uint32, vp, vp, C.c_uint32, vp, vp, vp,
                                  C.POINTER(PxcError)]),
    "pxc_sq_search_device": (C.c_int32, [vp, vp, C.c_uint32, C.c_uint32, C.c_uint32, vp, vp, C.c_uint32, vp, vp,
                                         vp, vp, C.POINTER(PxcError)]),
    "pxc_sq_last_scan_ms": (C.c_float, [vp]),
    "pxc_sq_last_accepted": (C.c_uint64, [vp]),
    "pxc_sq_last_fallback": (C.c_uint32, [vp]),
    "pxc_sq_last_retried": (C.c_uint32, [vp]),
}

_lib = None


def load() -> C.CDLL:
    """Load the CUDA library (once). Raises if it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m proxima_b200.build`; "
                "there is no CPU fallback for the device path")
        lib = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def call(name: str, *args) -> None:
    """Invoke a status-returning entry point and raise the mapped ProximaError."""
    err = PxcError()
    status = getattr(load(), name)(*args, C.byref(err))
    if status != 0:
        raise_for_status(status, err.a, err.b, err.parameter.decode(errors="replace"),
                         err.detail.decode(errors="replace"))


def ptr(arr) -> int | None:
    """Address of a numpy array or torch tensor (None passes through). The caller
    keeps `arr` alive until the call that uses the address returns."""
    if arr is None:
        return None
    if hasattr(arr, "data_ptr"):
        return arr.data_ptr()
    return arr.ctypes.data
