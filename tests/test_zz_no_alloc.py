"""The no-allocation MatMulNBits entry point (ort_cuda_matmul_nbits_noalloc).

Some hosts cannot call cudaMalloc once they are running (a device-memory
budget fixed at start-up, memory owned by another runtime's allocator, or a
latency path that cannot take cudaMalloc's implicit device synchronisation).
This entry point keeps its split-K scratch (needed by the shapes whose
cluster plan does not fit in shared memory) in a static device array of the
library.  The test calls it through the C ABI on device buffers and checks
it against the regular entry point on two calls in a row; the file is named
to be collected last.
"""
import ctypes

import numpy as np
import pytest

from tests.conftest import max_rel

pytestmark = pytest.mark.gpu

TOL = 1e-5  # exact-mode bar used by every GPU parity test


@pytest.mark.parametrize("K,N,bs,zp,M", [
    (4096, 3000, 128, True, 1),     # cluster plan: no scratch needed
    (14336, 1024, 128, True, 4),    # 28 chunks, M = 4
    (512, 777, 32, False, 2),       # single chunk: no scratch needed
    (2048, 128256 // 2, 128, True, 1),  # many tiles: no scratch needed
    (40960, 4096, 128, True, 3),    # cluster inbox too large: split-K, partials
                                    # in the static array
])
def test_noalloc_matches_regular_entry_point(K, N, bs, zp, M):
    from onnx_runtime_dart_b200 import CudaSession, DeviceTensor, _lib
    from onnx_runtime_dart_b200.workloads import make_nbits_weight
    L = _lib.load()
    rng = np.random.default_rng(K + N + M)
    B, sc, z = make_nbits_weight(rng, K, N, bs, zero_points=zp, scale_dtype=np.float16)
    with CudaSession(0) as s:
        s.upload_nbits("w", B, sc, z, k=K, n=N, block_size=bs)
        A = DeviceTensor.from_host(s, rng.standard_normal((M, K)).astype(np.float32))
        ref = s.matmul_nbits("w", A).numpy()
        Y = DeviceTensor(s, (M, N))
        for _ in range(2):
            before = s.launch_count()
            rc = L.ort_cuda_matmul_nbits_noalloc(s.handle, b"w", A.ptr, M, Y.ptr)
            assert rc == 0, _lib.last_error()
            s.sync()
            # one GEMV launch, plus the chunk-sum launch for split-K shapes
            assert s.launch_count() in (before + 1, before + 2)
            assert max_rel(ref, Y.numpy()) <= TOL


def test_noalloc_rejects_what_it_cannot_hold():
    from onnx_runtime_dart_b200 import CudaSession, DeviceTensor, _lib
    from onnx_runtime_dart_b200.workloads import make_nbits_weight
    L = _lib.load()
    rng = np.random.default_rng(3)
    K, N = 40960, 4096  # split-K, M=4: 80 chunks x 4 x 4096 partial floats > 2^20
    B, sc, z = make_nbits_weight(rng, K, N, 128, zero_points=False, scale_dtype=np.float16)
    with CudaSession(0) as s:
        s.upload_nbits("big", B, sc, z, k=K, n=N, block_size=128)
        A = DeviceTensor(s, (4, K))
        Y = DeviceTensor(s, (4, N))
        rc = L.ort_cuda_matmul_nbits_noalloc(s.handle, b"big", A.ptr, 4, Y.ptr)
        assert rc == _lib.ERR_INVALID_ARG
        assert "static scratch" in _lib.last_error()
        rc = L.ort_cuda_matmul_nbits_noalloc(s.handle, b"big", A.ptr, 1, Y.ptr)
        assert rc == 0, _lib.last_error()
        s.sync()
        rc = L.ort_cuda_matmul_nbits_noalloc(s.handle, b"big", A.ptr, 5, Y.ptr)
        assert rc == _lib.ERR_INVALID_ARG
        rc = L.ort_cuda_matmul_nbits_noalloc(s.handle, b"nope", A.ptr, 1, Y.ptr)
        assert rc == _lib.ERR_NOT_FOUND
