"""Device ArgMax / ArgMin over the last axis (ort_cuda_argmax): the greedy
selection step after the lm_head of a decode graph.

Parity is exact (integer output) against the oracle's restatement of
opArgMinMax (lib/src/onnx_ops.dart:2198-2237), which is itself pinned to
the reference's ORT fixtures (tests/test_oracle.py).  Cases cover the tie
rules (first index, or last with select_last_index), NaN (skipped, except
as a row's first element), infinities and signed zeros, rows of one and of
many 16K-column segments, and the lm_head -> ArgMax chain on device.
"""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def sess():
    from onnx_runtime_dart_b200 import CudaSession
    s = CudaSession(0)
    yield s
    s.close()


@pytest.mark.parametrize("case", ["argmax_axis1", "argmax_nan", "argmin_nokeep_last"])
def test_argmax_reference_fixtures(sess, golden, case):
    g = golden(case)
    a = g["meta"]["attrs"]
    axis, keepdims = int(a.get("axis", 0)), bool(a.get("keepdims", 1))
    is_max, last = g["meta"]["op_type"] == "ArgMax", bool(a.get("select_last_index", 0))
    x = g["in_x"]
    ax = axis + x.ndim if axis < 0 else axis
    got = sess.argmax(np.moveaxis(x, ax, -1), is_min=not is_max, select_last=last)
    if keepdims:
        got = np.expand_dims(got, ax)
    assert np.array_equal(got, g["expected"])


def _planted(rng, rows, cols):
    x = rng.standard_normal((rows, cols)).astype(np.float32)
    for r in range(rows):
        kind = r % 6
        if kind == 1:  # a tie of the maximum at three places
            idx = rng.choice(cols, size=min(3, cols), replace=False)
            x[r, idx] = x[r].max() + 1.0
        elif kind == 2:  # NaNs everywhere but the first element
            x[r, rng.choice(cols, size=max(1, cols // 7))] = np.nan
            x[r, 0] = 0.0
        elif kind == 3:  # a NaN first element
            x[r, 0] = np.nan
        elif kind == 4:  # +inf twice and -inf
            x[r, rng.integers(cols)] = np.inf
            x[r, rng.integers(cols)] = np.inf
            x[r, rng.integers(cols)] = -np.inf
        elif kind == 5:  # signed zeros as the extreme values
            x[r] = -np.abs(x[r]) - 1.0
            x[r, rng.choice(cols, size=min(2, cols), replace=False)] = -0.0
            x[r, rng.integers(cols)] = 0.0
    return x


@pytest.mark.parametrize("rows,cols", [(1, 1), (6, 7), (12, 1000), (6, 16384), (6, 16385),
                                       (3, 128256)])
@pytest.mark.parametrize("is_min,last", [(False, False), (False, True), (True, False),
                                         (True, True)])
def test_argmax_matches_oracle(sess, rows, cols, is_min, last):
    rng = np.random.default_rng(rows * 1000 + cols)
    x = _planted(rng, rows, cols)
    want = O.argminmax(x, axis=-1, keepdims=False, is_max=not is_min, select_last=last)
    got = sess.argmax(x, is_min=is_min, select_last=last)
    assert got.dtype == np.int64
    assert np.array_equal(got, want)
    # and again: the per-row tickets of the multi-segment path start from zero
    assert np.array_equal(sess.argmax(x, is_min=is_min, select_last=last), want)


def test_argmax_on_device_after_lm_head(sess):
    """Greedy decode step: lm_head GEMV into a device tensor, ArgMax on the
    device, only the indices read back; equals the oracle's ArgMax of the
    same logits."""
    import torch
    from onnx_runtime_dart_b200.workloads import make_nbits_weight
    rng = np.random.default_rng(8)
    K, N, M = 4096, 128256, 4
    B, sc, z = make_nbits_weight(rng, K, N, 128, zero_points=True, scale_dtype=np.float16)
    sess.upload_nbits("lm", B, sc, z, k=K, n=N, block_size=128)
    a = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).cuda()
    logits = sess.matmul_nbits("lm", a)
    idx = sess.argmax(logits)
    torch.cuda.synchronize()
    assert idx.dtype == torch.int64 and idx.device.type == "cuda"
    want = O.argminmax(logits.cpu().numpy(), axis=-1, keepdims=False)
    assert np.array_equal(idx.cpu().numpy(), want)
    sess.drop_weight("lm")


def test_argmax_rejects_empty_rows(sess):
    from onnx_runtime_dart_b200 import _lib
    L = _lib.load()
    out = np.zeros(2, np.int64)
    x = np.zeros((2, 1), np.float32)
    rc = L.ort_cuda_argmax(sess.handle, x.ctypes.data, 2, 0, 1, out.ctypes.data, _lib.HOST_IO)
    assert rc == _lib.ERR_INVALID_ARG
    rc = L.ort_cuda_argmax(sess.handle, x.ctypes.data, 2, 4, 2, out.ctypes.data, _lib.HOST_IO)
    assert rc == _lib.ERR_INVALID_ARG
