"""onnx_runtime_dart_b200 — B200-native MatMulNBits / MatMul / Gemm.

The product is libort_cuda.so (C ABI, include/ort_cuda.h) with hand-written
sm_100a kernels.  This package holds its sources (csrc/), the in-tree
build (build.py) and a Python mirror of the reference's operator interface
(session.py) used by the tests and the benchmark.
"""
from ._lib import StateError, UnsupportedError  # noqa: F401
from .session import (CudaSession, DeviceTensor, default_session, op_gemm,  # noqa: F401
                      op_matmul, op_matmul_nbits)

__version__ = "0.1.0"
