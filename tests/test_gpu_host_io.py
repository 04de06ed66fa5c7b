"""ORT_CUDA_HOST_IO calls of ort_cuda_matmul_nbits (the Dart binding's call:
host A in, host Y out) against the same op on device buffers, bit for bit.

At decode sizes (M <= 64) in the exact and strict modes the kernels store Y
straight into the host buffer through its device mapping: the caller's own
buffer when it is pinned, else the session's pinned staging, copied out on
the host after the wait.  Larger M and the MMA modes copy Y back from the
device.  Every combination must give the device call's bits.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

K, N, BS = 2048, 5000, 128


@pytest.fixture(scope="module")
def sess():
    from onnx_runtime_dart_b200 import CudaSession
    from onnx_runtime_dart_b200.workloads import make_nbits_weight
    rng = np.random.default_rng(31)
    B, sc, z = make_nbits_weight(rng, K, N, BS, zero_points=True, scale_dtype=np.float16)
    s = CudaSession(0)
    s.upload_nbits("w", B, sc, z, k=K, n=N, block_size=BS)
    yield s
    s.close()


def _host_call(s, A, Y, M, flags):
    from onnx_runtime_dart_b200 import _lib
    L = _lib.load()
    rc = L.ort_cuda_matmul_nbits(ctypes.c_void_p(s.handle), b"w", A, M, Y, flags | _lib.HOST_IO)
    _lib.check(rc, "ort_cuda_matmul_nbits")


@pytest.mark.parametrize("mode", ["exact", "strict", "mma_f16"])
@pytest.mark.parametrize("M", [1, 3, 16, 64, 65, 300])
def test_host_io_equals_device(sess, M, mode):
    import torch
    from onnx_runtime_dart_b200 import _lib
    if mode == "mma_f16" and M < 64:
        pytest.skip("the MMA mode is for prefill sizes")
    flags = _lib.flags_mode(_lib.MODES[mode])
    a = torch.randn(M, K, generator=torch.Generator().manual_seed(M))
    ref = sess.matmul_nbits("w", a.cuda(), flags=flags)
    torch.cuda.synchronize()
    ref = ref.cpu()
    # pageable host buffers: staged through the session's pinned memory
    a_np = a.numpy().copy()
    y_np = np.full((M, N), np.nan, np.float32)
    _host_call(sess, a_np.ctypes.data, y_np.ctypes.data, M, flags)
    assert np.array_equal(y_np, ref.numpy())
    # pinned host buffers: Y written in place at decode sizes
    a_p = a.clone().pin_memory()
    y_p = torch.full((M, N), float("nan")).pin_memory()
    _host_call(sess, a_p.data_ptr(), y_p.data_ptr(), M, flags)
    assert torch.equal(y_p, ref)
    # the same pinned output again (nothing left over from the first call)
    y_p.fill_(float("nan"))
    _host_call(sess, a_p.data_ptr(), y_p.data_ptr(), M, flags)
    assert torch.equal(y_p, ref)
