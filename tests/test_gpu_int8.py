"""MatMulInteger on tensor cores (ort_cuda_matmul_integer): the int8
dynamic-quantisation path of quantised LLMs (opMatMulInteger,
lib/src/onnx_qlinear_ops.dart:26-79).  Integer results: exact equality with
the oracle's restatement, itself pinned to the reference's ORT fixtures."""
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


@pytest.mark.parametrize("case", ["matmulinteger_nozp", "matmulinteger_percol_bzp",
                                  "matmulinteger_u8i8", "matmulinteger_batched"])
def test_matmul_integer_reference_fixtures(sess, golden, case):
    g = golden(case)
    a, b = g["init_a"], g["init_b"]
    az, bz = g.get("init_az"), g.get("init_bz")
    want = g["expected"]
    if b.ndim == 3:  # per-batch weights: one upload per batch
        for i in range(b.shape[0]):
            sess.upload_int8("fx", b[i], bz)
            assert np.array_equal(sess.matmul_integer("fx", a[i], az), want[i])
    else:
        sess.upload_int8("fx", b, bz)
        assert np.array_equal(sess.matmul_integer("fx", a, az), want)
    sess.drop_weight("fx")


def _rand(rng, shape, signed):
    return (rng.integers(-128, 128, shape) if signed else rng.integers(0, 256, shape)).astype(
        np.int8 if signed else np.uint8)


@pytest.mark.parametrize("M,K,N", [(1, 4096, 6144), (4, 2048, 1000), (16, 1000, 777),
                                   (100, 4096, 512), (300, 1536, 2048), (2048, 4096, 1024)])
@pytest.mark.parametrize("a_signed,b_signed,zps", [(False, True, "scalar"),
                                                   (False, False, "per"),
                                                   (True, True, None)])
def test_matmul_integer_matches_oracle(sess, M, K, N, a_signed, b_signed, zps):
    rng = np.random.default_rng(M + K + N)
    a = _rand(rng, (M, K), a_signed)
    b = _rand(rng, (K, N), b_signed)
    az = bz = None
    if zps == "scalar":
        az, bz = _rand(rng, (1,), a_signed), _rand(rng, (1,), b_signed)
    elif zps == "per":
        az, bz = _rand(rng, (M,), a_signed), _rand(rng, (N,), b_signed)
    sess.upload_int8("w8", b, bz)
    got = sess.matmul_integer("w8", a, az)
    want = O.matmul_integer(a, b, az, bz)
    assert got.dtype == np.int32
    assert np.array_equal(got.astype(np.int64), want)
    sess.drop_weight("w8")


def test_matmul_integer_on_device(sess):
    """Device tensors in and out, the zero point a device scalar (as
    DynamicQuantizeLinear leaves it); two calls in a row give the same bits
    (the K-split slices add into a zeroed output)."""
    import torch
    rng = np.random.default_rng(9)
    M, K, N = 1, 14336, 4096
    a = _rand(rng, (M, K), False)
    b = _rand(rng, (K, N), True)
    bz = _rand(rng, (N,), True)
    sess.upload_int8("dev", b, bz)
    ad = torch.from_numpy(a).cuda()
    zd = torch.tensor([117], dtype=torch.uint8, device="cuda")
    y1 = sess.matmul_integer("dev", ad, zd)
    y2 = sess.matmul_integer("dev", ad, zd)
    want = O.matmul_integer(a, b, np.array([117], np.uint8), bz)
    assert np.array_equal(y1.cpu().numpy().astype(np.int64), want)
    assert torch.equal(y1, y2)
    sess.drop_weight("dev")


def test_dynamic_quantize_linear_fixture(sess, golden):
    g = golden("dynamicquantizelinear")
    y, scale, zp = sess.dynamic_quantize_linear(g["in_x"])
    assert np.array_equal(y.astype(np.int64), g["expected_out0"])
    assert np.float32(scale) == np.float32(g["expected_out1"])
    assert zp == int(g["expected_out2"])


def _dql_cases():
    rng = np.random.default_rng(12)
    halves = np.arange(0, 511, dtype=np.float32) / 2  # 0, 0.5, ... 255: scale 1, ties to even
    return {
        "halves": halves,
        "zeros": np.zeros(1000, np.float32),
        "positive": np.abs(rng.standard_normal(4096)).astype(np.float32) + 0.25,
        "negative": -np.abs(rng.standard_normal(3000)).astype(np.float32) - 1.0,
        "one": np.array([3.25], np.float32),
        "wide": (rng.standard_normal(65536) * 7).astype(np.float32),
    }


@pytest.mark.parametrize("name", list(_dql_cases()))
def test_dynamic_quantize_linear_matches_oracle(sess, name):
    x = _dql_cases()[name]
    y, scale, zp = sess.dynamic_quantize_linear(x)
    wy, ws, wz = O.dynamic_quantize_linear(x)
    assert np.float32(scale) == ws and zp == wz
    assert np.array_equal(y, wy)


def test_int8_chain_on_device(sess):
    """x -> DynamicQuantizeLinear -> MatMulInteger(y, W, y_zp, W_zp), all on
    the device (the zero point never leaves it), equals the oracle chain."""
    import torch
    rng = np.random.default_rng(21)
    M, K, N = 4, 4096, 3000
    x = (rng.standard_normal((M, K)) * 3).astype(np.float32)
    b = _rand(rng, (K, N), True)
    bz = _rand(rng, (1,), True)
    sess.upload_int8("chain", b, bz)
    y, sc, zp = sess.dynamic_quantize_linear(torch.from_numpy(x).cuda())
    out = sess.matmul_integer("chain", y, zp)
    wy, ws, wz = O.dynamic_quantize_linear(x)
    want = O.matmul_integer(wy, b, np.array([wz], np.uint8), bz)
    assert float(sc.cpu()) == ws
    assert np.array_equal(out.cpu().numpy().astype(np.int64), want)
    sess.drop_weight("chain")
