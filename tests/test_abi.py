"""The C-ABI library: it loads, exports every symbol include/ort_cuda.h
declares, and validates arguments without touching a GPU."""
import ctypes
import os
import re
import subprocess

import pytest

from onnx_runtime_dart_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "ort_cuda.h")


def declared_symbols():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"ORT_CUDA_API\s+[^;(]*?\b(ort_cuda_\w+)\s*\(", src, re.S)))


def test_header_declares_the_binding_table():
    assert declared_symbols() == sorted(_lib.SIGNATURES)


def test_library_exports_every_declared_symbol():
    L = _lib.load()
    for name in declared_symbols():
        assert hasattr(L, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = sorted(set(re.findall(r" T (ort_cuda_\w+)", out)))
    assert exported == declared_symbols()


def test_library_links_no_torch_or_python():
    out = subprocess.run(["ldd", _lib.LIB_PATH], capture_output=True, text=True).stdout
    assert "torch" not in out and "python" not in out.lower()


def test_version_and_error_text():
    L = _lib.load()
    assert b"sm_100a" in L.ort_cuda_version()
    assert L.ort_cuda_device_count(None) == _lib.ERR_INVALID_ARG
    assert "NULL" in _lib.last_error()


def test_null_session_is_rejected():
    L = _lib.load()
    assert L.ort_cuda_set_mode(None, 0) == _lib.ERR_INVALID_ARG
    assert L.ort_cuda_sync(None) == _lib.ERR_INVALID_ARG
    assert L.ort_cuda_matmul_nbits(None, b"w", None, 1, None, 0) == _lib.ERR_INVALID_ARG
    assert L.ort_cuda_upload_nbits(None, b"w", None, None, None, 32, 8, 4, 32, 0) == \
        _lib.ERR_INVALID_ARG
    assert L.ort_cuda_close(None) == _lib.OK


def test_open_rank_validates_before_device():
    L = _lib.load()
    h = ctypes.c_void_p()
    assert L.ort_cuda_open_rank(0, 2, 2, None, 0, 1000, ctypes.byref(h)) == _lib.ERR_INVALID_ARG
    assert L.ort_cuda_open_rank(0, 0, 2, None, 0, 1000, ctypes.byref(h)) == _lib.ERR_INVALID_ARG
    assert L.ort_cuda_open_rank(0, 0, 1, None, 0, 0, ctypes.byref(h)) == _lib.ERR_INVALID_ARG


def test_open_without_gpu_reports_error():
    L = _lib.load()
    n = ctypes.c_int(-1)
    assert L.ort_cuda_device_count(ctypes.byref(n)) == _lib.OK
    if n.value > 0:
        pytest.skip("a GPU is visible")
    h = ctypes.c_void_p()
    rc = L.ort_cuda_open(0, 0, ctypes.byref(h))
    assert rc == _lib.ERR_CUDA and h.value is None
    assert "no CUDA device" in _lib.last_error()


def test_status_maps_to_reference_exceptions():
    with pytest.raises(_lib.UnsupportedError):
        _lib.check(_lib.ERR_UNSUPPORTED)
    with pytest.raises(_lib.StateError):
        _lib.check(_lib.ERR_TIMEOUT)
    with pytest.raises(ValueError):
        _lib.check(_lib.ERR_INVALID_ARG)
