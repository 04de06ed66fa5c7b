"""MatMulNBits with ArgMax fused into the decode GEMV
(ort_cuda_matmul_nbits_argmax): the greedy step after lm_head.

The fused path returns, for every row, the index that opArgMinMax
(lib/src/onnx_ops.dart:2198-2237, restated by the oracle) picks on the
logits this same call produces: exact integer parity against the oracle's
scan over the returned logits, and against ort_cuda_argmax on the logits of
a plain ort_cuda_matmul_nbits call.  Cases: every GEMV work plan (tile-major,
clusters, split-K), row counts that take one and several GEMV passes,
planted ties (duplicated weight columns, first or last index), a NaN
column 0 and non-finite rows, ArgMin, host buffers, and the unfused
fallbacks (STRICT mode, M > 64).
"""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

K, N, BS = 4096, 128256, 128


@pytest.fixture(scope="module")
def lm():
    from onnx_runtime_dart_b200 import CudaSession
    from onnx_runtime_dart_b200.workloads import make_nbits_weight
    rng = np.random.default_rng(21)
    B, sc, z = make_nbits_weight(rng, K, N, BS, zero_points=True, scale_dtype=np.float16)
    # duplicated columns give exactly tied logits: 7 = 1000 = 90000, 55 = 128255
    nb = K // BS
    zn = np.stack([z & 0xF, z >> 4], 1).ravel()[:N * nb].copy()
    for src, dst in ((7, 1000), (7, 90000), (55, 128255)):
        B[dst] = B[src]
        sc[dst * nb:(dst + 1) * nb] = sc[src * nb:(src + 1) * nb]
        zn[dst * nb:(dst + 1) * nb] = zn[src * nb:(src + 1) * nb]
    z = (zn[0::2] | (zn[1::2] << 4)).astype(np.uint8)
    s = CudaSession(0)
    s.upload_nbits("lm", B, sc, z, k=K, n=N, block_size=BS)
    yield s, (B, sc, z)
    s.close()


def _check(s, A, is_min=False, last=False, flags=0):
    import torch
    a = torch.from_numpy(A).cuda()
    idx, y = s.matmul_nbits_argmax("lm", a, is_min=is_min, select_last=last, logits=True,
                                   flags=flags)
    y_plain = s.matmul_nbits("lm", a, flags=flags)
    sep = s.argmax(y_plain, is_min=is_min, select_last=last)
    torch.cuda.synchronize()
    yn = y.cpu().numpy()
    assert np.array_equal(yn, y_plain.cpu().numpy(), equal_nan=True)
    want = O.argminmax(yn, axis=-1, keepdims=False, is_max=not is_min, select_last=last)
    assert np.array_equal(idx.cpu().numpy(), want)
    assert np.array_equal(sep.cpu().numpy(), want)
    return idx.cpu().numpy(), yn


@pytest.mark.parametrize("M", [1, 3, 8, 13])
def test_fused_argmax_every_plan(lm, M):
    s, _ = lm
    rng = np.random.default_rng(M)
    A = rng.standard_normal((M, K)).astype(np.float32)
    m = min(M, 8)
    _check(s, A)  # the first call times the plans
    # every candidate plan of the pass size gives the same logits and index
    for plan in range(16):
        try:
            s.set_gemv_plan("lm", m, plan)
        except ValueError:  # past the last candidate
            break
        _check(s, A)
    s.set_gemv_plan("lm", m, -1)


def test_fused_argmax_ties_and_variants(lm):
    s, (B, sc, z) = lm
    rng = np.random.default_rng(5)
    A = rng.standard_normal((4, K)).astype(np.float32)
    # make column 7 (and its copies 1000, 90000) the maximum of row 0 and
    # column 55 (copy 128255) the minimum of row 1: put A along the
    # dequantised column
    w7 = O.dequant_nbits(B[7:8], sc[7 * (K // BS):8 * (K // BS)].astype(np.float32),
                         None, K, 1, BS)
    A[0] = (w7[:, 0] / np.abs(w7).max() * 3.0).astype(np.float32)
    idx, y = _check(s, A)
    if y[0, 7] == y[0].max():
        assert idx[0] == 7
    idx_last, _ = _check(s, A, last=True)
    if y[0, 7] == y[0].max():
        assert idx_last[0] == 90000
    _check(s, A, is_min=True)
    _check(s, A, is_min=True, last=True)


def test_fused_argmax_non_finite_rows(lm):
    s, _ = lm
    rng = np.random.default_rng(6)
    A = rng.standard_normal((3, K)).astype(np.float32)
    A[1, 17] = np.nan   # every logit of the row is NaN: column 0 is NaN -> 0
    A[2, 99] = np.inf   # this path gives NaN across such a row too -> 0
    idx, y = _check(s, A)
    assert idx[1] == 0 and idx[2] == 0
    assert np.isnan(y[1]).all()


def test_fused_argmax_host_buffers_and_fallbacks(lm):
    from onnx_runtime_dart_b200 import _lib
    s, _ = lm
    rng = np.random.default_rng(7)
    A = rng.standard_normal((2, K)).astype(np.float32)
    idx, y = s.matmul_nbits_argmax("lm", A, logits=True)
    assert np.array_equal(idx, O.argminmax(y, axis=-1, keepdims=False))
    idx2 = s.matmul_nbits_argmax("lm", A)  # no logits wanted
    assert np.array_equal(idx, idx2)
    # STRICT (the reference's rounding, no fused path) and M > 64
    _check(s, A, flags=_lib.flags_mode(_lib.MODE_STRICT))
    A70 = rng.standard_normal((70, K)).astype(np.float32)
    import torch
    a = torch.from_numpy(A70).cuda()
    idx = s.matmul_nbits_argmax("lm", a)
    want = s.argmax(s.matmul_nbits("lm", a))
    assert torch.equal(idx, want)
