"""ctypes binding of libort_cuda.so (declared in include/ort_cuda.h).

The library is built in-tree by ``python -m onnx_runtime_dart_b200.build``
(or ``__graft_entry__.build()``).  Loading fails loudly when it is missing:
there is no fallback implementation behind this package.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libort_cuda.so")

# status codes (ort_cuda.h)
OK = 0
ERR_INVALID_ARG = 1
ERR_UNSUPPORTED = 2
ERR_CUDA = 3
ERR_NCCL = 4
ERR_TIMEOUT = 5
ERR_NOT_FOUND = 6
ERR_OOM = 7

# modes
MODE_EXACT = 0
MODE_STRICT = 1
MODE_MMA_F16 = 2
MODE_MMA_BF16 = 3
MODES = {"exact": MODE_EXACT, "strict": MODE_STRICT, "mma_f16": MODE_MMA_F16,
         "mma_bf16": MODE_MMA_BF16}

# call flags
HOST_IO = 0x1
TRANS_A = 0x2
MODE_OVERRIDE = 0x100


def flags_mode(m: int) -> int:
    return MODE_OVERRIDE | ((m & 0xF) << 12)


# upload flags
SCALES_F32 = 0
SCALES_F16 = 1
ZP_FLAT = 0x0
ZP_PER_COLUMN = 0x10
ARG_MIN = 0x20  # ort_cuda_argmax flags
ARG_SELECT_LAST = 0x40
ROTARY = 0x80  # attention flags
ROTARY_INTERLEAVED = 0x200
ROTARY_BHSD = 0x400
TOPK_SMALLEST = 0x800
FUSE_DROP_PARTS = 0x1  # ort_cuda_fuse_nbits flags

# Every symbol include/ort_cuda.h declares, with (restype, argtypes).
_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_f = ctypes.c_float
_cp = ctypes.c_char_p
SIGNATURES = {
    "ort_cuda_last_error": (ctypes.c_char_p, []),
    "ort_cuda_version": (ctypes.c_char_p, []),
    "ort_cuda_device_count": (_int, [ctypes.POINTER(_int)]),
    "ort_cuda_open": (_int, [_int, _int, ctypes.POINTER(_vp)]),
    "ort_cuda_nccl_unique_id": (_int, [_vp]),
    "ort_cuda_open_rank": (_int, [_int, _int, _int, _vp, _int, _int, ctypes.POINTER(_vp)]),
    "ort_cuda_close": (_int, [_vp]),
    "ort_cuda_set_mode": (_int, [_vp, _int]),
    "ort_cuda_set_stream": (_int, [_vp, _vp]),
    "ort_cuda_sync": (_int, [_vp]),
    "ort_cuda_rank_info": (_int, [_vp, ctypes.POINTER(_int), ctypes.POINTER(_int)]),
    "ort_cuda_upload_nbits": (_int, [_vp, _cp, _vp, _vp, _vp, _i64, _i64, _int, _int, _int]),
    "ort_cuda_upload_nbits_file": (_int, [_vp, _cp, _cp, _i64, _i64, _i64, _i64, _i64, _int,
                                          _int, _int]),
    "ort_cuda_upload_dense": (_int, [_vp, _cp, _vp, _i64, _i64, _int]),
    "ort_cuda_drop_weight": (_int, [_vp, _cp]),
    "ort_cuda_weight_shape": (_int, [_vp, _cp, ctypes.POINTER(_i64), ctypes.POINTER(_i64)]),
    "ort_cuda_alloc": (_int, [_vp, _i64, ctypes.POINTER(_vp)]),
    "ort_cuda_free": (_int, [_vp, _vp]),
    "ort_cuda_h2d": (_int, [_vp, _vp, _vp, _i64]),
    "ort_cuda_d2h": (_int, [_vp, _vp, _vp, _i64]),
    "ort_cuda_matmul_nbits": (_int, [_vp, _cp, _vp, _i64, _vp, _int]),
    "ort_cuda_matmul_nbits_noalloc": (_int, [_vp, _cp, _vp, _i64, _vp]),
    "ort_cuda_matmul": (_int, [_vp, _cp, _vp, _i64, _vp, _int]),
    "ort_cuda_gemm": (_int, [_vp, _cp, _vp, _i64, _vp, _i64, _i64, _f, _f, _vp, _int]),
    "ort_cuda_matmul_batched": (_int, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _int]),
    "ort_cuda_gemv_plan_get": (_int, [_vp, _cp, _int, ctypes.POINTER(_int)]),
    "ort_cuda_gemv_plan_set": (_int, [_vp, _cp, _int, _int]),
    "ort_cuda_argmax": (_int, [_vp, _vp, _i64, _i64, _i64, _vp, _int]),
    "ort_cuda_upload_int8": (_int, [_vp, _cp, _vp, _i64, _i64, _int, _vp, _i64]),
    "ort_cuda_dynamic_quantize_linear": (_int, [_vp, _vp, _i64, _vp, _vp, _vp, _int]),
    "ort_cuda_matmul_integer": (_int, [_vp, _cp, _vp, _i64, _int, _vp, _i64, _vp, _int]),
    "ort_cuda_launch_count": (_int, [_vp, ctypes.POINTER(_i64)]),
    "ort_cuda_topk": (_int, [_vp, _vp, _i64, _i64, _i64, _i64, _vp, _vp, _int]),
    "ort_cuda_slice_last_seq": (_int, [_vp, _vp, _i64, _i64, _i64, _vp, _int]),
    "ort_cuda_group_query_attention": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64,
                                              _int, _int, _i64, ctypes.c_double, _vp, _vp, _i64,
                                              _i64, _vp, _i64, _i64, _i64, _vp, _vp, _vp, _int]),
    "ort_cuda_multi_head_attention": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _int, _i64,
                                             ctypes.c_double, _vp, _i64, _i64, _vp, _int]),
    "ort_cuda_fused_sdpa": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64,
                                   _i64, ctypes.c_double, _vp, _int]),
    "ort_cuda_rotary_embedding": (_int, [_vp, _vp, _vp, _int, _vp, _vp, _i64, _i64, _i64, _i64,
                                         _i64, _i64, _i64, _vp, _int]),
    "ort_cuda_graph_begin": (_int, [_vp]),
    "ort_cuda_graph_end": (_int, [_vp, ctypes.POINTER(_int)]),
    "ort_cuda_graph_launch": (_int, [_vp, _int]),
    "ort_cuda_graph_drop": (_int, [_vp, _int]),
    "ort_cuda_profile_enable": (_int, [_vp, _int]),
    "ort_cuda_profile_reset": (_int, [_vp]),
    "ort_cuda_profile_read": (_int, [_vp, _int, _cp, _int, ctypes.POINTER(_i64),
                                     ctypes.POINTER(ctypes.c_double)]),
    "ort_cuda_probe_ffma": (_int, [_vp, ctypes.POINTER(ctypes.c_double)]),
    "ort_cuda_matmul_nbits_argmax": (_int, [_vp, _cp, _vp, _i64, _vp, _vp, _int]),
    "ort_cuda_set_peer_wait": (_int, [_vp, _int]),
    "ort_cuda_set_replicate_bytes": (_int, [_vp, _i64]),
    "ort_cuda_weight_columns": (_int, [_vp, _cp, ctypes.POINTER(_i64), ctypes.POINTER(_i64)]),
    "ort_cuda_fuse_nbits": (_int, [_vp, _cp, ctypes.POINTER(_cp), _int, _int]),
    "ort_cuda_matmul_nbits_group": (_int, [_vp, _cp, _vp, _i64, ctypes.POINTER(_vp), _int]),
}

_lib = None


class UnsupportedError(NotImplementedError):
    """Dart's UnsupportedError (onnx_qlinear_ops.dart:117-119)."""


class StateError(RuntimeError):
    """Dart's StateError (onnx_graph.dart:789-795); carries the status code."""

    def __init__(self, msg: str, code: int = ERR_CUDA):
        super().__init__(msg)
        self.code = code


def load():
    """Loads libort_cuda.so; raises ImportError if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -m onnx_runtime_dart_b200.build` "
            "(there is no non-CUDA implementation of this path)")
    L = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def last_error() -> str:
    return load().ort_cuda_last_error().decode(errors="replace")


def check(rc: int, what: str = "") -> None:
    """Maps a status to the reference's exception types."""
    if rc == OK:
        return
    msg = f"{what}: {last_error()}" if what else last_error()
    if rc == ERR_UNSUPPORTED:
        raise UnsupportedError(msg)
    if rc == ERR_INVALID_ARG:
        raise ValueError(msg)
    if rc == ERR_NOT_FOUND:
        raise KeyError(msg)
    raise StateError(msg, rc)
