"""Host mirror of proxima-quantize on the B200 backend.

``kmeans`` keeps the reference's interface (crates/proxima-quantize/src/kmeans.rs:59-65:
a flat ``n * dim`` array, ``dim``, ``k``, ``max_iterations`` and a seeded
ChaCha8 stream) and returns the same ``Clustering`` (centroids, inertia,
iterations). The work runs on the GPU through ``pxc_kmeans``; there is no CPU
path. An explicit ``init`` replaces k-means++ seeding (an option the reference
does not have; the Lloyd iterations are the same).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _native as N


@dataclass
class Clustering:
    """crates/proxima-quantize/src/kmeans.rs:36-48."""

    centroids: np.ndarray  # (k, dim) float32
    inertia: float
    iterations: int
    assignment: np.ndarray | None = None  # (n,) uint32, the last assignment pass
    path: int = 0  # 0 exact CUDA-core assignment, 1 tensor-core screening + exact re-scoring
    reseeded: int = 0
    rescanned: int = 0
    screen_passes: int = 0
    screen_ms: float = 0.0


def kmeans(points, dim: int, k: int, max_iterations: int, seed: int = 0, init=None,
           context=None, want_assignment: bool = False) -> Clustering:
    """``kmeans(points, dim, k, max_iterations, &mut ChaCha8Rng::seed_from_u64(seed))``.

    ``points`` is a flat or (n, dim) float32 array on the host, or a CUDA torch
    tensor (then the device entry point runs on the current stream).
    """
    from .index import Context

    ctx = context or Context.default()
    is_torch = hasattr(points, "is_cuda") and points.is_cuda
    if is_torch:
        import torch

        pts = points.contiguous().view(-1)
        n = pts.numel() // dim if dim else 0
        kk = max(min(k, n), 1)
        cent = torch.empty((kk, dim), dtype=torch.float32, device=pts.device)
        assign = torch.empty((max(n, 1),), dtype=torch.int32, device=pts.device) if want_assignment else None
        d_init = None
        if init is not None:
            d_init = torch.as_tensor(init, dtype=torch.float32, device=pts.device).contiguous().view(-1)
            if d_init.numel() < kk * dim:
                raise ValueError("init holds fewer than k * dim values")
        info = N.PxcKmeansInfo()
        N.call("pxc_kmeans_device", ctx.handle, pts.data_ptr(), n, dim, k, max_iterations,
               None if d_init is None else d_init.data_ptr(), seed, cent.data_ptr(),
               None if assign is None else assign.data_ptr(), C.byref(info),
               torch.cuda.current_stream(pts.device).cuda_stream)
        return Clustering(cent.cpu().numpy(), info.inertia, info.iterations,
                          None if assign is None else assign[:n].cpu().numpy().view(np.uint32),
                          info.path, info.reseeded, info.rescanned, info.screen_passes, info.screen_ms)
    pts = np.ascontiguousarray(points, dtype=np.float32).reshape(-1)
    n = pts.size // dim if dim else 0
    kk = max(min(k, n), 1)
    cent = np.zeros((kk, dim), dtype=np.float32)
    assign = np.zeros(max(n, 1), dtype=np.uint32) if want_assignment else None
    init_arr = None
    if init is not None:
        init_arr = np.ascontiguousarray(init, dtype=np.float32).reshape(-1)
        if init_arr.size < kk * dim:
            raise ValueError("init holds fewer than k * dim values")
    info = N.PxcKmeansInfo()
    N.call("pxc_kmeans", ctx.handle, N.ptr(pts), n, dim, k, max_iterations, N.ptr(init_arr), seed,
           N.ptr(cent), N.ptr(assign), C.byref(info))
    return Clustering(cent, info.inertia, info.iterations,
                      None if assign is None else assign[:n], info.path, info.reseeded, info.rescanned,
                      info.screen_passes, info.screen_ms)
