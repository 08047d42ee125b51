"""Snapshots of an IVF-PQ index in the reference's file format, loaded and
saved straight between the file image and the device.

The format is crates/proxima-store/src/snapshot.rs (version 1) over the codec
of crates/proxima-store/src/codec.rs. ``load_ivfpq`` is ``decode`` for an
IVF-PQ body and ``save_ivfpq`` is ``encode``: the large arrays (vectors,
codes, list assignments, centroids, codebooks) move by one copy each between
the image and the index's device buffers and their CRC-32C is computed on the
device (pxc_ivfpq_snapshot_load / _save). Metadata is the codec's section,
encoded and decoded here (codec.rs:170-200, 367-392).
``write_snapshot`` / ``read_snapshot`` are the atomic file steps of
snapshot.rs:518-560.
"""
from __future__ import annotations

import ctypes as C
import os
import struct
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

from . import _native as N
from .errors import Corruption, Io

KIND_FLAT, KIND_HNSW, KIND_IVFPQ = 1, 2, 3
_KINDS = {KIND_FLAT: "flat", KIND_HNSW: "hnsw", KIND_IVFPQ: "ivfpq"}
_TAG_TEXT, _TAG_INT, _TAG_FLOAT, _TAG_BOOL = 1, 2, 3, 4


@dataclass
class IvfPqConfig:
    """IvfPqConfig (crates/proxima-index/src/ivfpq.rs:104-150) with the
    reference's defaults: nprobe max(nlist / 16, 1), rerank 0, seed 0x1FF9C0D,
    25 iterations, a 100 000-vector training sample, train_threshold 100 * nlist,
    retain_vectors on."""
    nlist: int
    subspaces: int
    nprobe: int | None = None
    rerank: int = 0
    seed: int = 0x1FF_9C0D
    max_iterations: int = 25
    training_sample: int = 100_000
    train_threshold: int | None = None
    retain_vectors: bool = True

    def __post_init__(self):
        if self.nprobe is None:
            self.nprobe = max(self.nlist // 16, 1)
        if self.train_threshold is None:
            self.train_threshold = self.nlist * 100

    def to_native(self) -> N.PxcIvfpqConfig:
        c = N.PxcIvfpqConfig()
        sat = lambda v: min(int(v), 0xFFFFFFFF)  # codec.rs len_prefix saturates
        c.nlist, c.subspaces, c.nprobe, c.rerank = sat(self.nlist), sat(self.subspaces), sat(self.nprobe), sat(self.rerank)
        c.seed = int(self.seed) & 0xFFFFFFFFFFFFFFFF
        c.max_iterations, c.training_sample = sat(self.max_iterations), sat(self.training_sample)
        c.train_threshold = min(int(self.train_threshold), 0xFFFFFFFFFFFFFFFF)
        c.retain_vectors = 1 if self.retain_vectors else 0
        return c

    @classmethod
    def from_native(cls, c: N.PxcIvfpqConfig) -> "IvfPqConfig":
        return cls(c.nlist, c.subspaces, c.nprobe, c.rerank, c.seed, c.max_iterations, c.training_sample,
                   c.train_threshold, bool(c.retain_vectors))


_REPORT_FIELDS = ("sampled", "coarse_inertia", "coarse_iterations", "residual_inertia", "populated_lists",
                  "largest_list")


@dataclass
class SnapshotInfo:
    """What a snapshot says about itself (snapshot.rs:96-110, plus the IVF-PQ body's small fields)."""
    format_version: int
    kind: str
    dim: int
    metric: int
    body_bytes: int
    nslots: int
    len: int
    config: IvfPqConfig | None = None
    trained: bool = False
    lists: int = 0
    has_vectors: bool = False
    report: dict | None = None
    metadata_offset: int = 0
    metadata_bytes: int = 0
    extra: dict = field(default_factory=dict)

    @classmethod
    def from_native(cls, i: N.PxcSnapshotInfo) -> "SnapshotInfo":
        out = cls(i.format_version, _KINDS.get(i.kind, str(i.kind)), i.dim, i.metric, i.body_bytes, i.nslots, i.live)
        if i.kind == KIND_IVFPQ:
            out.config = IvfPqConfig.from_native(i.config)
            out.trained, out.lists, out.has_vectors = bool(i.trained), i.lists, bool(i.has_vectors)
            out.report = {f: getattr(i.report, f) for f in _REPORT_FIELDS} if i.has_report else None
            out.metadata_offset, out.metadata_bytes = i.metadata_offset, i.metadata_bytes
        return out


def crc32c(data, crc: int = 0) -> int:
    """crc32c_append (crates/proxima-store/src/crc.rs:64-79) over host bytes."""
    buf = memoryview(data).cast("B")
    if len(buf) == 0:
        return crc
    arr = np.frombuffer(buf, dtype=np.uint8)
    return int(N.load().pxc_crc32c_append(crc, arr.ctypes.data, len(arr)))


def crc32c_device(tensor, context=None) -> int:
    """CRC-32C of a CUDA tensor's bytes, computed on the device."""
    from .index import Context

    ctx = context or Context.default()
    out = C.c_uint32()
    nbytes = tensor.numel() * tensor.element_size()
    N.call("pxc_crc32c_device", ctx.handle, tensor.data_ptr() if nbytes else None, nbytes, C.byref(out), None)
    return out.value


# ---- metadata section (codec.rs) ----

def _encode_value(out: list, v) -> None:
    if isinstance(v, bool):
        out.append(struct.pack("<BB", _TAG_BOOL, 1 if v else 0))
    elif isinstance(v, (int, np.integer)):
        out.append(struct.pack("<BQ", _TAG_INT, int(v) & 0xFFFFFFFFFFFFFFFF))
    elif isinstance(v, (float, np.floating)):
        out.append(struct.pack("<Bd", _TAG_FLOAT, float(v)))
    elif isinstance(v, str):
        b = v.encode("utf-8")
        out.append(struct.pack("<BI", _TAG_TEXT, len(b)) + b)
    else:
        raise TypeError(f"unsupported metadata value {v!r}")


def encode_metadata(metadata, nslots: int) -> bytes:
    """The metadata section for `nslots` slots: a u32 count, then per slot the
    codec's Metadata with its keys in byte order (codec.rs:170-200). `metadata`
    is a list of dicts (None or {} for none), or None for none anywhere."""
    if metadata is None:
        return struct.pack("<I", nslots) + bytes(4 * nslots)
    if len(metadata) != nslots:
        raise ValueError(f"{len(metadata)} metadata entries for {nslots} slots")
    out = [struct.pack("<I", nslots)]
    for m in metadata:
        if not m:
            out.append(b"\0\0\0\0")
            continue
        out.append(struct.pack("<I", len(m)))
        for key in sorted(m, key=lambda k: k.encode("utf-8")):
            kb = key.encode("utf-8")
            out.append(struct.pack("<I", len(kb)) + kb)
            _encode_value(out, m[key])
    return b"".join(out)


def decode_metadata(image, offset: int = 0, nbytes: int | None = None) -> list[dict]:
    """The metadata section at `offset` of `image` as a list of dicts (codec.rs:367-392)."""
    mv = memoryview(image).cast("B")
    end = len(mv) if nbytes is None else offset + nbytes
    pos = offset

    def take(n):
        nonlocal pos
        if end - pos < n:
            raise Corruption("metadata", f"truncated at byte {pos}: wanted {n} more, {end - pos} remain")
        b = mv[pos:pos + n]
        pos += n
        return b

    def u32():
        return struct.unpack("<I", take(4))[0]

    def text():
        n = u32()
        return bytes(take(n)).decode("utf-8")

    count = u32()
    out = []
    for _ in range(count):
        nf = u32()
        m = {}
        for _ in range(nf):
            key = text()
            tag = take(1)[0]
            if tag == _TAG_TEXT:
                m[key] = text()
            elif tag == _TAG_INT:
                m[key] = struct.unpack("<q", take(8))[0]
            elif tag == _TAG_FLOAT:
                m[key] = struct.unpack("<d", take(8))[0]
            elif tag == _TAG_BOOL:
                m[key] = take(1)[0] != 0
            else:
                raise Corruption("metadata", f"metadata value tag {tag} is not one of 1..=4")
        out.append(m)
    return out


# ---- images ----

def peek(image) -> SnapshotInfo:
    """Header, checksum, space and kind of a snapshot image (snapshot.rs:271-299); an
    IVF-PQ body is checked in full."""
    arr = np.frombuffer(memoryview(image).cast("B"), dtype=np.uint8)
    info = N.PxcSnapshotInfo()
    N.call("pxc_snapshot_peek", arr.ctypes.data if len(arr) else None, len(arr), C.byref(info))
    return SnapshotInfo.from_native(info)


def load_ivfpq(image, context=None, with_metadata: bool = True):
    """decode (snapshot.rs:192-269) of an IVF-PQ snapshot image into a new
    device IvfPqIndex. Returns (index, info); with `with_metadata` the index
    carries the decoded per-slot metadata for filtered searches."""
    from .core import Metric
    from .index import Context
    from .ivfpq import IvfPqIndex

    ctx = context or Context.default()
    arr = np.frombuffer(memoryview(image).cast("B"), dtype=np.uint8)
    h = N.vp()
    info = N.PxcSnapshotInfo()
    N.call("pxc_ivfpq_snapshot_load", ctx.handle, arr.ctypes.data if len(arr) else None, len(arr), C.byref(h),
           C.byref(info))
    out = SnapshotInfo.from_native(info)
    idx = IvfPqIndex.adopt(h, ctx, out.dim, out.lists, out.config.subspaces, Metric(out.metric), out.nslots)
    idx.config = out.config
    idx.report = out.report
    if with_metadata:
        idx.set_metadata(decode_metadata(arr, out.metadata_offset, out.metadata_bytes))
    return idx, out


def save_ivfpq(index, config: IvfPqConfig | None = None, report: dict | None = None, metadata=None) -> bytearray:
    """encode (snapshot.rs:120-200) of a device IvfPqIndex, as a bytearray. `config` defaults to
    the index's own (or IvfPqConfig(nlist, subspaces)); `report` to the one its
    training produced; `metadata` to the per-slot metadata it holds."""
    cfg = config or getattr(index, "config", None) or IvfPqConfig(index.nlist, index.m)
    rep = report if report is not None else getattr(index, "report", None)
    meta = metadata if metadata is not None else getattr(index, "_metadata", None)
    section = encode_metadata(meta, index.nslots) if meta is not None else None
    sec = None if section is None else np.frombuffer(section, dtype=np.uint8)
    native_cfg = cfg.to_native()
    native_rep = None
    if rep is not None:
        native_rep = N.PxcIvfpqReport()
        for f in _REPORT_FIELDS:
            setattr(native_rep, f, rep[f])
    need = C.c_uint64()
    args = (index.handle, C.byref(native_cfg), C.byref(native_rep) if native_rep is not None else None,
            N.ptr(sec), 0 if sec is None else len(sec))
    N.call("pxc_ivfpq_snapshot_save", *args, None, 0, C.byref(need))
    out = bytearray(need.value)
    buf = (C.c_char * need.value).from_buffer(out)
    N.call("pxc_ivfpq_snapshot_save", *args, C.addressof(buf), need.value, C.byref(need))
    del buf  # releases the export so the bytearray can be resized by its owner
    return out


def write_snapshot(path, image) -> int:
    """write_snapshot (snapshot.rs:518-560): `path`.tmp, fsync, rename over
    `path`, fsync of the directory. Returns the bytes written."""
    path = Path(path)
    tmp = path.with_suffix(".tmp")
    try:
        with open(tmp, "wb") as f:
            f.write(image)
            f.flush()
            os.fsync(f.fileno())
    except OSError as e:
        raise Io("write snapshot", str(tmp), str(e)) from e
    try:
        os.replace(tmp, path)
    except OSError as e:
        raise Io("rename snapshot", str(path), str(e)) from e
    try:
        fd = os.open(path.parent if str(path.parent) else ".", os.O_RDONLY)
    except OSError:
        fd = None
    if fd is not None:
        try:
            os.fsync(fd)
        except OSError as e:
            raise Io("sync snapshot directory", str(path.parent), str(e)) from e
        finally:
            os.close(fd)
    return len(image)


def read_snapshot(path) -> bytes:
    """The image at `path` (read_snapshot, snapshot.rs:562-569)."""
    try:
        return Path(path).read_bytes()
    except OSError as e:
        raise Io("read snapshot", str(path), str(e)) from e
