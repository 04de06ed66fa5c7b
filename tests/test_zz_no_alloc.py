"""The no-allocation MatMulNBits entry point (ort_cuda_matmul_nbits_noalloc).

Some hosts cannot call cudaMalloc once they are running (a device-memory
budget fixed at start-up, memory owned by another runtime's allocator, or a
latency path that cannot take cudaMalloc's implicit device synchronisation).
This entry point keeps its split-K scratch (needed by the shapes whose
cluster plan does not fit in shared memory) in a static device array of the
library.  The tests call it through the C ABI on device buffers and check it
against the regular entry point on two calls in a row, bit for bit (every
GEMV work plan gives the same bits).  The file is named to be collected
last; its first test relies on no earlier no-allocation call in the process.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_noalloc_first_call_refused_inside_a_capture():
    """The first call on a device looks up the static array's address, which
    may load the module and so must not happen inside a stream capture: it
    returns an error instead (no other test of this process calls the entry
    point before this one)."""
    from onnx_runtime_dart_b200 import CudaSession, DeviceTensor, _lib
    from onnx_runtime_dart_b200.workloads import make_nbits_weight
    L = _lib.load()
    rng = np.random.default_rng(11)
    K, N = 1024, 512
    B, sc, z = make_nbits_weight(rng, K, N, 128, zero_points=True, scale_dtype=np.float16)
    with CudaSession(0) as s:
        s.upload_nbits("w", B, sc, z, k=K, n=N, block_size=128)
        A = DeviceTensor.from_host(s, rng.standard_normal((1, K)).astype(np.float32))
        Y = DeviceTensor(s, (1, N))
        ref = s.matmul_nbits("w", A).numpy()
        s.graph_begin()
        rc = L.ort_cuda_matmul_nbits_noalloc(s.handle, b"w", A.ptr, 1, Y.ptr)
        msg = _lib.last_error()
        gid = s.graph_end()
        s.graph_drop(gid)
        assert rc == _lib.ERR_INVALID_ARG, msg
        assert "capture" in msg
        # outside a capture the same call sets the device up and runs
        rc = L.ort_cuda_matmul_nbits_noalloc(s.handle, b"w", A.ptr, 1, Y.ptr)
        assert rc == 0, _lib.last_error()
        s.sync()
        assert np.array_equal(ref, Y.numpy())


@pytest.mark.parametrize("K,N,bs,zp,M", [
    (4096, 3000, 128, True, 1),     # cluster plan: no scratch needed
    (14336, 1024, 128, True, 4),    # 28 chunks, M = 4
    (512, 777, 32, False, 2),       # single chunk: no scratch needed
    (2048, 128256 // 2, 128, True, 1),  # many tiles: no scratch needed
    (40960, 4096, 128, True, 3),    # cluster inbox too large: split-K, partials
                                    # in the static array
    (40960, 4096, 128, False, 4),   # split-K would need 80 x 4 x 4096 partial
                                    # floats (> 2^20): a plan that fits runs
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
            assert np.array_equal(ref, Y.numpy())


def test_noalloc_rejects_what_it_cannot_run():
    from onnx_runtime_dart_b200 import CudaSession, DeviceTensor, _lib
    from onnx_runtime_dart_b200.workloads import make_nbits_weight
    L = _lib.load()
    rng = np.random.default_rng(3)
    K, N = 2048, 512
    B, sc, z = make_nbits_weight(rng, K, N, 128, zero_points=False, scale_dtype=np.float16)
    with CudaSession(0) as s:
        s.upload_nbits("w", B, sc, z, k=K, n=N, block_size=128)
        A = DeviceTensor(s, (5, K))
        Y = DeviceTensor(s, (5, N))
        rc = L.ort_cuda_matmul_nbits_noalloc(s.handle, b"w", A.ptr, 5, Y.ptr)
        assert rc == _lib.ERR_INVALID_ARG
        assert "M <= 4" in _lib.last_error()
        rc = L.ort_cuda_matmul_nbits_noalloc(s.handle, b"nope", A.ptr, 1, Y.ptr)
        assert rc == _lib.ERR_NOT_FOUND
    # a STRICT session's regular entry point reproduces the reference's
    # rounding; the no-allocation call does not, so it refuses
    with CudaSession(0, mode="strict") as s:
        s.upload_nbits("w", B, sc, z, k=K, n=N, block_size=128)
        A = DeviceTensor(s, (1, K))
        Y = DeviceTensor(s, (1, N))
        rc = L.ort_cuda_matmul_nbits_noalloc(s.handle, b"w", A.ptr, 1, Y.ptr)
        assert rc == _lib.ERR_UNSUPPORTED
        assert "STRICT" in _lib.last_error()
