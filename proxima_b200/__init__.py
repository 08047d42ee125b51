"""proxima_b200 — B200-native backend for Proxima's nearest-neighbour hot path.

The product is ``lib/libproxima_cuda.so`` (sm_100a kernels behind the C ABI in
``include/proxima_cuda.h``). This package is the host-side mirror of the
reference's Rust API for that path (VectorIndex / FlatIndex / recall_at_k),
calling the C ABI through ctypes.
"""
from .core import MAX_K, Metric, SearchResult, VectorSpace
from .errors import (Capacity, Configuration, Corruption, DeviceTimeout, DimensionMismatch,
                     DuplicateId, Internal, NonFinite, ProximaError, UnknownId)

__all__ = [
    "MAX_K", "Metric", "SearchResult", "VectorSpace",
    "ProximaError", "DimensionMismatch", "UnknownId", "DuplicateId", "Capacity", "NonFinite",
    "Corruption", "Configuration", "Internal", "DeviceTimeout",
    "AcceptAll", "Context", "FlatIndex", "IndexStats", "RecallReport", "recall_at_k",
]


def __getattr__(name):
    # The device-facing classes load the CUDA library on first use only, so
    # importing the package (and its pure-host helpers) works without a GPU.
    if name in ("AcceptAll", "Context", "FlatIndex", "IndexStats", "RecallReport", "recall_at_k"):
        from . import index
        return getattr(index, name)
    raise AttributeError(name)
