"""Exact-mode decode GEMV on the activations where its arithmetic is fragile.

The tensor-core GEMV (csrc/gemv_tc.cu) multiplies the int4 weights with a
fixed-point copy of A: per 512-k chunk and row, X = rint(a * 2^S) with the
largest |a| of that chunk at 2^22, so an outlier channel leaves the other
elements of its chunk fewer significant bits.  Real decoder hidden states
have such channels, 10^2 - 10^4 times the median.  These tests hold the
path to the exact mode's bar, row by row (max|dY_row| / max|Y_ref_row| <=
1e-5), against the oracle's restatement of the reference's arithmetic
(lib/src/onnx_qlinear_ops.dart:120-155, lib/src/gemm_kernel_simd.dart), at
the shapes of the Qwen3-0.6B sweep (bs 32, fp32 scales, zero points) and the
Llama-3-8B projections (bs 128, fp16 scales, zero points).

Rows holding an inf or a NaN are the one documented divergence: the
reference accumulates each output column on its own and gives +-inf or NaN
per column, while this path gives NaN for the whole row (its per-chunk
scale of the row is not finite).  test_non_finite_row_divergence pins that.
"""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

EXACT_TOL = 1e-5


@pytest.fixture(scope="module")
def sess():
    from onnx_runtime_dart_b200 import CudaSession
    s = CudaSession(0, mode="exact")
    yield s
    s.close()


def _row(rng, K, kind):
    a = rng.standard_normal(K).astype(np.float32)
    if kind == "outlier_1e2":
        a[rng.choice(K, size=4, replace=False)] *= 100.0
    elif kind == "outlier_1e4":
        a[rng.choice(K, size=3, replace=False)] = rng.choice([-1.0, 1.0], 3) * 1e4
    elif kind == "outlier_mixed":  # 10^2 .. 10^4 channels spread over the row
        idx = rng.choice(K, size=8, replace=False)
        a[idx] = (rng.choice([-1.0, 1.0], 8) * 10.0 ** rng.uniform(2, 4, 8)).astype(np.float32)
    elif kind == "scale_up40":
        a *= np.float32(2.0 ** 40)
    elif kind == "scale_down40":
        a *= np.float32(2.0 ** -40)
    elif kind == "one_chunk_large":  # large values inside one 512-k chunk only
        c = rng.integers(0, max(1, K // 512))
        a[c * 512:(c + 1) * 512] *= 1e3
    elif kind == "all_positive":
        a = np.abs(a)
    elif kind == "tiny_and_huge_chunks":  # chunk magnitudes 2^-30 .. 2^30
        for c in range(0, K, 512):
            a[c:c + 512] *= np.float32(2.0 ** rng.integers(-30, 31))
    return a


KINDS = ["outlier_1e2", "outlier_1e4", "outlier_mixed", "scale_up40", "scale_down40",
         "one_chunk_large", "all_positive", "tiny_and_huge_chunks"]

SHAPES = [  # (K, N, block size, scale dtype)
    (1024, 2048, 32, np.float32),      # cfg3 q
    (3072, 1024, 32, np.float32),      # cfg3 down
    (4096, 6144, 128, np.float16),     # cfg5 qkv
    (14336, 4096, 128, np.float16),    # cfg5 down
]


def _check_rows(ref, y):
    for r in range(ref.shape[0]):
        den = np.abs(ref[r].astype(np.float64)).max()
        err = np.abs(ref[r].astype(np.float64) - y[r]).max()
        assert den > 0 and err / den <= EXACT_TOL, (r, err / den)


@pytest.mark.parametrize("K,N,bs,sdt", SHAPES)
@pytest.mark.parametrize("M", [1, 3, 8])
def test_fragile_activations(sess, K, N, bs, sdt, M):
    rng = np.random.default_rng(K * 3 + N + M)
    B, s, z = O.make_nbits_weight(rng, K, N, bs, zero_points=True, scale_dtype=sdt)
    sess.upload_nbits("w", B, s, z, k=K, n=N, block_size=bs)
    s32 = s.astype(np.float32)
    for i in range(0, len(KINDS), M):
        kinds = [KINDS[(i + j) % len(KINDS)] for j in range(M)]
        A = np.stack([_row(rng, K, k) for k in kinds])
        y = sess.matmul_nbits("w", A)
        ref = O.matmul_nbits(A, B, s32, z, K, N, 4, bs, threads=8)
        _check_rows(ref, y)
    sess.drop_weight("w")


def test_cfg3_lm_head_outliers(sess):
    """The 151936-column lm_head of the Qwen3-0.6B sweep with outlier rows."""
    K, N, bs = 1024, 151936, 32
    rng = np.random.default_rng(77)
    B, s, z = O.make_nbits_weight(rng, K, N, bs, zero_points=True)
    sess.upload_nbits("lm", B, s, z, k=K, n=N, block_size=bs)
    A = np.stack([_row(rng, K, k) for k in ("outlier_1e4", "outlier_mixed", "all_positive")])
    y = sess.matmul_nbits("lm", A)
    ref = O.matmul_nbits(A, B, s, z, K, N, 4, bs, threads=8)
    _check_rows(ref, y)
    sess.drop_weight("lm")


@pytest.mark.parametrize("bad", [np.inf, -np.inf, np.nan])
def test_non_finite_row_divergence(sess, bad):
    """A row holding inf or NaN: this path returns NaN across the row (the
    reference gives +-inf or NaN per column), and the other rows of the same
    call are unaffected."""
    K, N, bs = 4096, 1024, 128
    rng = np.random.default_rng(5)
    B, s, z = O.make_nbits_weight(rng, K, N, bs, zero_points=True, scale_dtype=np.float16)
    sess.upload_nbits("w", B, s, z, k=K, n=N, block_size=bs)
    A = rng.standard_normal((3, K)).astype(np.float32)
    A[1, 1234] = bad
    y = sess.matmul_nbits("w", A)
    ref = O.matmul_nbits(A, B, s.astype(np.float32), z, K, N, 4, bs, threads=8)
    assert np.isnan(y[1]).all()
    if not np.isnan(bad):
        # the reference's per-column result keeps infinities where this path
        # has NaN: that is the divergence
        assert np.isinf(ref[1]).any()
    _check_rows(ref[[0, 2]], y[[0, 2]])
    sess.drop_weight("w")
