"""The C ABI without a GPU: libcairn_b200.so loads, exports every entry include/cairn_b200.h declares, and answers
the reference's guards (shape, view, disjointness) with statuses before it touches the device."""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import cairn_b200
from cairn_b200 import _lib


def test_every_declared_entry_is_exported():
    declared = cairn_b200.header_symbols()
    assert len(declared) >= 16
    handle = C.CDLL(str(cairn_b200.LIB_PATH))
    missing = [name for name in declared if not hasattr(handle, name)]
    assert not missing, missing
    assert set(declared) == set(_lib.SIGNATURES), "the ctypes signatures cover exactly the header"


def test_version_and_status_strings():
    lib = cairn_b200.lib()
    assert lib.cairn_b200_version() == 100
    for s in range(9):
        assert lib.cairn_b200_status_string(s)
    assert lib.cairn_b200_status_string(0) == b"ok"


def _bufs():
    c = np.zeros(6, np.float32)
    a = np.zeros(6, np.uint16)
    b = np.zeros(9, np.uint16)
    return c, a, b


def test_the_extents_are_checked_against_the_views():
    """cr::tensor::shape (runtime/cairn_tensor.hpp:22-24): a 2x3x3 multiply whose b holds 6, not 9, elements traps
    in the reference (tests/soundness/test_tensor.py:103-114); here it is ERR_SHAPE and nothing is queued."""
    lib = cairn_b200.lib()
    c, a, b = _bufs()
    assert lib.cairn_b200_mma_bf16(None, 2, 3, 3, c.ctypes.data, 6, a.ctypes.data, 6, b.ctypes.data, 6) == _lib.ERR_SHAPE
    assert lib.cairn_b200_mma_bf16(None, 2, 3, 3, c.ctypes.data, 7, a.ctypes.data, 6, b.ctypes.data, 9) == _lib.ERR_SHAPE
    big = 1 << 40
    assert lib.cairn_b200_mma_bf16(None, big, big, 1, c.ctypes.data, 0, a.ctypes.data, 0, b.ctypes.data, 0) == _lib.ERR_SHAPE


def test_null_and_misaligned_views_are_refused():
    """cr::view (runtime/cairn_runtime.hpp:194-200): a null view of nonzero extent, or one off its alignment."""
    lib = cairn_b200.lib()
    c, a, b = _bufs()
    assert lib.cairn_b200_mma_bf16(None, 2, 3, 3, None, 6, a.ctypes.data, 6, b.ctypes.data, 9) == _lib.ERR_VIEW
    assert lib.cairn_b200_mma_bf16(None, 2, 3, 3, c.ctypes.data + 2, 6, a.ctypes.data, 6, b.ctypes.data, 9) == _lib.ERR_VIEW
    assert lib.cairn_b200_mma_bf16(None, 2, 3, 3, c.ctypes.data, 6, a.ctypes.data + 1, 6, b.ctypes.data, 9) == _lib.ERR_VIEW
    x = np.zeros(8, np.float32)
    assert lib.cairn_b200_saxpy_f32(None, 4, None, x.ctypes.data, x.ctypes.data, 1.0) == _lib.ERR_VIEW


def test_an_output_overlapping_an_input_is_refused():
    """cr::disjoint (runtime/cairn_runtime.hpp:201-205) on the cf_ entry's views."""
    lib = cairn_b200.lib()
    buf = np.zeros(64, np.float32)
    p = buf.ctypes.data
    assert lib.cairn_b200_mma_bf16(None, 2, 2, 2, p, 4, p + 8, 4, p + 64, 4) == _lib.ERR_OVERLAP
    # saxpy may run in place on x or y, but not on a shifted view of either
    assert lib.cairn_b200_saxpy_f32(None, 8, p + 4, p, p + 128, 2.0) == _lib.ERR_OVERLAP
    assert lib.cairn_b200_gemm(None, 0, 2, 2, 2, p, 0, p + 64, 0, p + 4, 0, None, 0) == _lib.ERR_OVERLAP


def test_arguments_outside_the_domain_are_refused():
    lib = cairn_b200.lib()
    buf = np.zeros(64, np.float32)
    p = buf.ctypes.data
    assert lib.cairn_b200_gemm(None, 9, 2, 2, 2, p, 0, p + 64, 0, p + 128, 0, None, 0) == _lib.ERR_ARG
    assert lib.cairn_b200_gemm(None, 0, 2, 2, 2, p, 0, p + 64, 0, p + 128, 7, None, 0) == _lib.ERR_ARG
    assert lib.cairn_b200_gemm(None, 0, 2, 2, 2, p, 0, p + 64, 0, p + 128, 2, None, 5) == _lib.ERR_ARG


def test_empty_multiplies_queue_nothing():
    """cr::tensor::launch returns before any launch when m or n is 0 (cairn_tensor.hpp:209), and a multiply with
    k == 0 adds no products: no device is touched, so these succeed without one."""
    lib = cairn_b200.lib()
    c, a, b = _bufs()
    assert lib.cairn_b200_mma_bf16(None, 0, 3, 3, c.ctypes.data, 0, a.ctypes.data, 0, b.ctypes.data, 9) == 0
    assert lib.cairn_b200_mma_bf16(None, 2, 3, 0, c.ctypes.data, 6, a.ctypes.data, 0, b.ctypes.data, 0) == 0


def test_the_package_fails_loudly_without_the_library(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "LIB_PATH", tmp_path / "missing.so")
    monkeypatch.setattr(_lib, "_lib", None)
    with pytest.raises(cairn_b200.CairnError):
        _lib.lib()
