"""Device TopK over the last axis (ort_cuda_topk) and the last-position
slice (ort_cuda_slice_last_seq): candidate selection after lm_head.

Parity is exact (indices and the selected values) against the oracle's
restatement of opTopK (lib/src/onnx_ops.dart:2261-2303), which is pinned to
the reference's ORT fixtures (tests/test_oracle.py): ties to the smaller
index, NaN ranked above every number, -0.0 equal to 0.0.
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


@pytest.mark.parametrize("case", ["topk_largest", "topk_smallest_axis0"])
def test_topk_reference_fixtures(sess, golden, case):
    g = golden(case)
    a = g["meta"]["attrs"]
    x, k = g["in_x"], int(g["init_k"].ravel()[0])
    ax = int(a.get("axis", -1))
    ax = ax + x.ndim if ax < 0 else ax
    v, i = sess.topk(np.moveaxis(x, ax, -1), k, largest=bool(a.get("largest", 1)))
    assert np.array_equal(np.moveaxis(v, -1, ax), g["expected_out0"])
    assert np.array_equal(np.moveaxis(i, -1, ax), g["expected_out1"])


def _planted(rng, rows, cols):
    x = rng.standard_normal((rows, cols)).astype(np.float32)
    for r in range(rows):
        kind = r % 5
        if kind == 1:  # many exact ties
            x[r] = np.round(x[r] * 2) / 2
        elif kind == 2:  # NaNs, infinities
            x[r, rng.choice(cols, size=max(1, cols // 9))] = np.nan
            x[r, rng.integers(cols)] = np.inf
            x[r, rng.integers(cols)] = -np.inf
        elif kind == 3:  # signed zeros at the top
            x[r] = -np.abs(x[r])
            x[r, rng.choice(cols, size=min(cols, 5), replace=False)] = -0.0
            x[r, rng.choice(cols, size=min(cols, 3), replace=False)] = 0.0
        elif kind == 4:  # all equal
            x[r] = 1.5
    return x


@pytest.mark.parametrize("rows,cols,k", [(1, 1, 1), (3, 7, 7), (5, 1000, 50), (5, 4096, 1024),
                                         (2, 128256, 40), (5, 3000, 1),
                                         # segmented rows at the largest k, and a
                                         # 256000-column row at its k limit (7
                                         # segments of 40960 columns, 7 x 585 <= 4096)
                                         (3, 128256, 1024), (2, 256000, 585)])
@pytest.mark.parametrize("largest", [True, False])
def test_topk_matches_oracle(sess, rows, cols, k, largest):
    rng = np.random.default_rng(rows * 131 + cols + k)
    x = _planted(rng, rows, cols)
    want_v, want_i = O.topk(x, k, largest=largest)
    v, i = sess.topk(x, k, largest=largest)
    assert i.dtype == np.int64
    assert np.array_equal(i, want_i)
    assert np.array_equal(v, want_v, equal_nan=True)
    v2, i2 = sess.topk(x, k, largest=largest)  # stateless: same again
    assert np.array_equal(i2, i)


def test_last_token_lm_head_topk_on_device(sess):
    """The lastTokenLogits path on the device: hidden [B, S, H] -> last
    position -> lm_head GEMV -> TopK; only B x k values and indices leave
    the GPU, and they equal the oracle's TopK of the same logits."""
    import torch
    from onnx_runtime_dart_b200.workloads import make_nbits_weight
    rng = np.random.default_rng(9)
    Bt, S, H, V, k = 2, 37, 2048, 128256, 50
    Bw, sc, z = make_nbits_weight(rng, H, V, 128, zero_points=False, scale_dtype=np.float16)
    sess.upload_nbits("lm", Bw, sc, None, k=H, n=V, block_size=128)
    hidden = torch.from_numpy(rng.standard_normal((Bt, S, H)).astype(np.float32)).cuda()
    last = sess.slice_last_seq(hidden)
    assert tuple(last.shape) == (Bt, 1, H)
    logits = sess.matmul_nbits("lm", last)
    v, i = sess.topk(logits, k)
    torch.cuda.synchronize()
    assert np.array_equal(last.cpu().numpy(), O.slice_last_seq(hidden.cpu().numpy()))
    want_v, want_i = O.topk(logits.cpu().numpy(), k)
    assert np.array_equal(i.cpu().numpy(), want_i)
    assert np.array_equal(v.cpu().numpy(), want_v)
    sess.drop_weight("lm")


def test_topk_rejects_bad_k(sess):
    from onnx_runtime_dart_b200 import UnsupportedError
    x = np.zeros((2, 10), np.float32)
    with pytest.raises(ValueError):
        sess.topk(x, 11)
    with pytest.raises(UnsupportedError):
        sess.topk(np.zeros((1, 2000), np.float32), 1025)
    # one past the segment limit of a 256000-column row (stated in ort_cuda.h)
    with pytest.raises(UnsupportedError, match="k <= 585"):
        sess.topk(np.zeros((1, 256000), np.float32), 586)
