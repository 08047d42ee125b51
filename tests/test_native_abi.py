"""CPU checks of the C-ABI library: it loads without a GPU and exports every declared symbol."""
import ctypes
import re
from pathlib import Path

import numpy as np

from proxima_b200 import _native, fixtures

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols() -> set[str]:
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names.update(re.findall(r"\b(pxc_[a-z0-9_]+)\s*\(", text))
    return names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_native.LIB_PATH))
    declared = declared_symbols()
    assert declared, "no declarations found in include/*.h"
    missing = [n for n in declared if not hasattr(lib, n)]
    assert not missing, missing
    # the Python binding table covers the whole header
    assert declared == set(_native.SIGNATURES), declared ^ set(_native.SIGNATURES)


def test_abi_version_and_no_gpu_error_path():
    lib = _native.load()
    assert lib.pxc_abi_version() >> 16 == 1
    # without a usable device, context creation fails with a status, not a crash
    import torch
    if not torch.cuda.is_available():
        err = _native.PxcError()
        handle = ctypes.c_void_p()
        dev = (ctypes.c_int * 1)(0)
        status = lib.pxc_ctx_create(dev, 1, ctypes.byref(handle), ctypes.byref(err))
        assert status != 0 and not handle.value


def test_fixtures_are_deterministic_and_slice_consistent():
    a = fixtures.blobs_u8(3000, 128, 64, 1, 2)
    b = fixtures.blobs_u8(1000, 128, 64, 1, 2, row_begin=2000)
    assert np.array_equal(a[2000:], b)
    assert np.all(a == np.floor(a)) and a.min() >= 0 and a.max() <= 255
    s1 = fixtures.sphere_blobs(500, 96, 32, 3, 4, 0.05)
    s2 = fixtures.sphere_blobs(500, 96, 32, 3, 4, 0.05)
    assert np.array_equal(s1, s2)
    assert np.allclose(np.linalg.norm(s1, axis=1), 1.0, atol=1e-5)
    q = fixtures.quickstart()
    assert q.shape == (5000, 64)
    assert q[0, 0] == 0.0  # sin(0) + 0


def test_host_mirror_rejects_like_the_reference():
    from proxima_b200.core import Metric, VectorSpace
    from proxima_b200.errors import Configuration, DimensionMismatch, NonFinite
    import pytest

    with pytest.raises(Configuration):
        VectorSpace(0, Metric.EUCLIDEAN)
    s = VectorSpace(3, Metric.EUCLIDEAN)
    with pytest.raises(DimensionMismatch):
        s.validate([1.0])
    with pytest.raises(NonFinite) as e:
        s.validate([1.0, float("inf"), 3.0])
    assert e.value.index == 1
    assert Configuration("k", 1, "x").is_caller_error()
