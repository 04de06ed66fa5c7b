"""MatMulNBits weights uploaded straight from an external-data file
(ort_cuda_upload_nbits_file), the path of models whose `.onnx.data` is too
large to read into host memory (the reference reads initializers on demand
through loadOnnxModel's resolve(), lib/onnx_runtime_dart_io.dart:19-45).

The file upload must give the same device weight as the in-memory upload:
results are compared bit for bit on the same activations.
"""
import numpy as np
import pytest

from oracle import oracle as O
from tests.conftest import max_rel

pytestmark = pytest.mark.gpu


def _write(path, parts, gap=13):
    """Writes the arrays back to back after `gap` filler bytes each (odd
    offsets, as tensors in a data file need not be aligned); returns the
    offset of each."""
    offs = []
    with open(path, "wb") as f:
        for a in parts:
            f.write(b"\x5a" * gap)
            offs.append(f.tell())
            f.write(np.ascontiguousarray(a).tobytes())
    return offs


@pytest.mark.parametrize("K,N,bs,f16,zp", [(4096, 6000, 128, True, True),
                                           (1000, 777, 32, False, True),
                                           (2048, 40000, 64, True, False)])
def test_file_upload_equals_memory_upload(tmp_path, K, N, bs, f16, zp):
    from onnx_runtime_dart_b200 import CudaSession
    rng = np.random.default_rng(K + N)
    B, s, z = O.make_nbits_weight(rng, K, N, bs, zero_points=zp,
                                  scale_dtype=np.float16 if f16 else np.float32)
    path = str(tmp_path / "model.onnx.data")
    offs = _write(path, [B, s] + ([z] if zp else []))
    A = rng.standard_normal((3, K)).astype(np.float32)
    with CudaSession(0) as sess:
        sess.upload_nbits("mem", B, s, z, k=K, n=N, block_size=bs)
        sess.upload_nbits_file("file", path, b_offset=offs[0], scales_offset=offs[1],
                               zp_offset=offs[2] if zp else None, k=K, n=N, block_size=bs,
                               scales_f16=f16)
        y_mem = sess.matmul_nbits("mem", A)
        y_file = sess.matmul_nbits("file", A)
    assert np.array_equal(y_mem, y_file)
    ref = O.matmul_nbits(A, B, s.astype(np.float32), z, K, N, 4, bs, threads=8)
    assert max_rel(ref, y_file) <= 1e-5


def test_file_upload_rejects_ranges_outside_the_file(tmp_path):
    from onnx_runtime_dart_b200 import CudaSession
    rng = np.random.default_rng(3)
    K, N, bs = 256, 64, 32
    B, s, z = O.make_nbits_weight(rng, K, N, bs, zero_points=True)
    path = str(tmp_path / "short.onnx.data")
    offs = _write(path, [B, s, z])
    with CudaSession(0) as sess:
        with pytest.raises(ValueError, match="outside"):
            sess.upload_nbits_file("w", path, b_offset=offs[0], scales_offset=offs[1],
                                   zp_offset=offs[2] + 1, k=K, n=N, block_size=bs)
        with pytest.raises(ValueError, match="outside"):
            sess.upload_nbits_file("w", path, b_offset=offs[0], scales_offset=offs[1],
                                   zp_offset=offs[2], k=K, n=N + 1, block_size=bs)
        with pytest.raises(ValueError, match="cannot open"):
            sess.upload_nbits_file("w", path + ".missing", b_offset=0, scales_offset=0,
                                   zp_offset=None, k=K, n=N, block_size=bs)
        assert "w" not in sess.weights
