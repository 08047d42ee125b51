"""Host mirror of proxima-quantize on the B200 backend.

``kmeans`` keeps the reference's interface (crates/proxima-quantize/src/kmeans.rs:59-65:
a flat ``n * dim`` array, ``dim``, ``k``, ``max_iterations`` and a
``&mut ChaCha8Rng``) and returns the same ``Clustering`` (centroids, inertia,
iterations); the generator is advanced in place, as the reference's is. The
work runs on the GPU through ``pxc_kmeans``; there is no CPU path. An explicit
``init`` replaces k-means++ seeding (an option the reference does not have; the
Lloyd iterations are the same).

``ProductQuantizer`` / ``DistanceTable`` mirror crates/proxima-quantize/src/product.rs
(train, encode, decode, distance_table, squared_l2 / inner_product) over
``pxc_pq_*``.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _native as N


class ChaCha8Rng:
    """rand_chacha 0.3.1's ChaCha8Rng as the boundary carries it (``pxc_rng``:
    seed, stream, word position). Draws run in the native library on the host."""

    def __init__(self, state: N.PxcRng):
        self._state = state

    @classmethod
    def seed_from_u64(cls, seed: int) -> "ChaCha8Rng":
        """rand_core 0.6.4 SeedableRng::seed_from_u64 (PCG32 expansion of the u64)."""
        st = N.PxcRng()
        N.call("pxc_rng_seed_from_u64", seed & (2**64 - 1), C.byref(st))
        return cls(st)

    @classmethod
    def from_seed(cls, seed: bytes, stream: int = 0, word_pos: int = 0) -> "ChaCha8Rng":
        """ChaCha8Rng::from_seed + set_stream + set_word_pos."""
        if len(seed) != 32:
            raise ValueError("a ChaCha8Rng seed is 32 bytes")
        st = N.PxcRng()
        C.memmove(st.seed, bytes(seed), 32)
        st.stream = stream
        st.word_pos_lo = word_pos & (2**64 - 1)
        st.word_pos_hi = word_pos >> 64
        return cls(st)

    def get_seed(self) -> bytes:
        return bytes(self._state.seed)

    def get_stream(self) -> int:
        return int(self._state.stream)

    def get_word_pos(self) -> int:
        return int(self._state.word_pos_hi) << 64 | int(self._state.word_pos_lo)

    def next_u32_array(self, n: int) -> np.ndarray:
        out = np.zeros(n, np.uint32)
        N.call("pxc_rng_next_u32", C.byref(self._state), N.ptr(out), n)
        return out

    def next_u32(self) -> int:
        return int(self.next_u32_array(1)[0])

    def gen_index(self, bound: int) -> int:
        """Rng::gen_range(0..bound) for usize."""
        out = C.c_uint64()
        N.call("pxc_rng_gen_index", C.byref(self._state), bound, C.byref(out))
        return int(out.value)

    def gen_f64(self, low: float, high: float) -> float:
        """Rng::gen_range(low..high) for f64."""
        out = C.c_double()
        N.call("pxc_rng_gen_f64", C.byref(self._state), low, high, C.byref(out))
        return float(out.value)

    @property
    def state(self) -> N.PxcRng:
        return self._state


def chacha_block(key, counter: int, stream: int, rounds: int) -> np.ndarray:
    """The ChaCha block function of the native library (16 u32 words)."""
    k = np.ascontiguousarray(key, np.uint32)
    if k.size != 8:
        raise ValueError("a ChaCha key is 8 words")
    out = np.zeros(16, np.uint32)
    N.call("pxc_chacha_block", N.ptr(k), counter, stream, rounds, N.ptr(out))
    return out


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


def kmeans(points, dim: int, k: int, max_iterations: int, rng: ChaCha8Rng | None = None, init=None,
           context=None, want_assignment: bool = False, seed: int | None = None) -> Clustering:
    """``kmeans(points, dim, k, max_iterations, &mut rng)``.

    ``rng`` is advanced in place by the k-means++ draws. ``seed`` is shorthand
    for a fresh ``ChaCha8Rng.seed_from_u64(seed)``. ``points`` is a flat or
    (n, dim) float32 array on the host, or a CUDA torch tensor (then the device
    entry point runs on the current stream).
    """
    from .index import Context

    if rng is None and init is None:
        rng = ChaCha8Rng.seed_from_u64(0 if seed is None else seed)
    rng_ptr = None if rng is None else C.byref(rng.state)
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
               None if d_init is None else d_init.data_ptr(), rng_ptr, cent.data_ptr(),
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
    N.call("pxc_kmeans", ctx.handle, N.ptr(pts), n, dim, k, max_iterations, N.ptr(init_arr), rng_ptr,
           N.ptr(cent), N.ptr(assign), C.byref(info))
    return Clustering(cent, info.inertia, info.iterations,
                      None if assign is None else assign[:n], info.path, info.reseeded, info.rescanned,
                      info.screen_passes, info.screen_ms)


def kmeans_sharded(points, dim: int, k: int, max_iterations: int, init, context) -> Clustering:
    """k-means over points sharded across the ranks of `context`'s communicator
    (pxc_kmeans_sharded): `points` is this rank's CUDA tensor (its consecutive range
    of the global point order), `init` the k x dim start shared by every rank.
    Returns the global centroids and this rank's assignment."""
    import torch

    pts = points.contiguous().view(-1)
    n = pts.numel() // dim
    d_init = torch.as_tensor(init, dtype=torch.float32, device=pts.device).contiguous().view(-1)
    kk = d_init.numel() // dim
    cent = torch.empty((kk, dim), dtype=torch.float32, device=pts.device)
    assign = torch.empty((n,), dtype=torch.int32, device=pts.device)
    info = N.PxcKmeansInfo()
    N.call("pxc_kmeans_sharded", context.handle, pts.data_ptr(), n, dim, k, max_iterations, d_init.data_ptr(),
           cent.data_ptr(), assign.data_ptr(), C.byref(info), torch.cuda.current_stream(pts.device).cuda_stream)
    return Clustering(cent[:info.k].cpu().numpy(), info.inertia, info.iterations,
                      assign.cpu().numpy().view(np.uint32), info.path, info.reseeded, info.rescanned,
                      info.screen_passes, info.screen_ms)


CENTROIDS_PER_SUBSPACE = 256


def pq_layout(dim: int, m: int) -> tuple[list[int], list[int]]:
    """Subspace widths and offsets (product.rs:227-238): widths differ by at most one, remainder leading."""
    base, rem = divmod(dim, m)
    widths = [base + (1 if s < rem else 0) for s in range(m)]
    offsets = [0]
    for w in widths:
        offsets.append(offsets[-1] + w)
    return widths, offsets


class DistanceTable:
    """product.rs:553-601: m x 256 squared-L2 and dot entries for one query."""

    def __init__(self, squared: np.ndarray, dot: np.ndarray):
        self.squared = squared  # (m, 256) float32
        self.dot = dot

    @property
    def subspaces(self) -> int:
        return self.squared.shape[0]

    def squared_l2(self, code) -> float:
        """product.rs:580-586: sequential f32 sum of the m looked-up entries."""
        s = np.float32(0.0)
        for sub, byte in enumerate(np.asarray(code, np.uint8)):
            s = np.float32(s + self.squared[sub, byte])
        return float(s)

    def inner_product(self, code) -> float:
        """product.rs:595-601: the negated sequential sum of the dot entries."""
        s = np.float32(0.0)
        for sub, byte in enumerate(np.asarray(code, np.uint8)):
            s = np.float32(s + self.dot[sub, byte])
        return float(-s)


class ProductQuantizer:
    """product.rs:162-182 on the GPU: ``codebooks`` 256 x dim float32, subspace-major."""

    def __init__(self, dim: int, subspaces: int, codebooks, training_inertia: float = 0.0,
                 training_iterations: int = 0, context=None):
        from .index import Context

        self.ctx = context or Context.default()
        self.dim = dim
        self.subspaces = subspaces
        self.codebooks = np.ascontiguousarray(codebooks, np.float32).reshape(-1)
        if self.codebooks.size != CENTROIDS_PER_SUBSPACE * dim:
            raise ValueError("codebooks hold 256 * dim floats")
        self.training_inertia = training_inertia
        self.training_iterations = training_iterations
        self.subspace_dims, self.offsets = pq_layout(dim, subspaces)

    @classmethod
    def train(cls, dim: int, training, subspaces: int, max_iterations: int = 25, seed: int = 0x5EED,
              context=None) -> "ProductQuantizer":
        """ProductQuantizer::train (product.rs:198-296) with PqConfig(subspaces, seed, max_iterations)."""
        from .index import Context

        ctx = context or Context.default()
        t = np.ascontiguousarray(training, np.float32).reshape(-1)
        n = t.size // dim if (dim and t.size % dim == 0) else 0
        books = np.zeros(CENTROIDS_PER_SUBSPACE * dim, np.float32)
        inertia = C.c_double()
        iters = C.c_uint64()
        N.call("pxc_pq_train", ctx.handle, N.ptr(t) if t.size else None, n, dim, subspaces, max_iterations,
               seed, N.ptr(books), C.byref(inertia), C.byref(iters))
        return cls(dim, subspaces, books, inertia.value, iters.value, ctx)

    @property
    def code_len(self) -> int:
        return self.subspaces

    def encode(self, vectors) -> np.ndarray:
        """encode_into (product.rs:361-380) for each row: (n, m) uint8."""
        v = np.ascontiguousarray(vectors, np.float32).reshape(-1, self.dim)
        out = np.zeros((v.shape[0], self.subspaces), np.uint8)
        N.call("pxc_pq_encode", self.ctx.handle, N.ptr(self.codebooks), self.dim, self.subspaces, N.ptr(v),
               v.shape[0], N.ptr(out))
        return out

    def decode(self, codes) -> np.ndarray:
        """decode (product.rs:387-398) for each code: (n, dim) float32."""
        c = np.ascontiguousarray(codes, np.uint8).reshape(-1, self.subspaces)
        out = np.zeros((c.shape[0], self.dim), np.float32)
        N.call("pxc_pq_decode", self.ctx.handle, N.ptr(self.codebooks), self.dim, self.subspaces, N.ptr(c),
               c.shape[0], N.ptr(out))
        return out

    def distance_tables(self, queries) -> tuple[np.ndarray, np.ndarray]:
        """distance_table (product.rs:407-439) for each query: (nq, m, 256) squared and dot arrays."""
        q = np.ascontiguousarray(queries, np.float32).reshape(-1, self.dim)
        sq = np.zeros((q.shape[0], self.subspaces, CENTROIDS_PER_SUBSPACE), np.float32)
        dot = np.zeros_like(sq)
        N.call("pxc_pq_tables", self.ctx.handle, N.ptr(self.codebooks), self.dim, self.subspaces, N.ptr(q),
               q.shape[0], N.ptr(sq), N.ptr(dot))
        return sq, dot

    def distance_table(self, query) -> DistanceTable:
        sq, dot = self.distance_tables(np.asarray(query, np.float32).reshape(1, self.dim))
        return DistanceTable(sq[0], dot[0])
