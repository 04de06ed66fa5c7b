"""Pins the CPU oracle (oracle/oracle.c) to the reference before any GPU
result is compared against it.

- every hot-path fixture of the reference's ORT-oracle suite
  (test/fixtures/matmulnbits_*, gemm_transB_bias, matmul_batched), with the
  reference's own tolerance (test/fixture_parity_test.dart:21, :242, :256);
- the hand-computed Gemm answer of test/gemm_prepack_test.dart:147;
- the fp16 widening values of test/loader_test.dart:78-87 plus all 65536
  fp16 patterns against IEEE conversion;
- the kernel shapes of test/gemm_kernel_test.dart:45-97;
- the column-split invariance of test/parallel_pool_test.dart (bitwise).
"""
import numpy as np
import pytest

from oracle import oracle as O
from tests.conftest import cosine

FIXTURE_TOL = 2e-5  # fixture_parity_test.dart:21


def _fixture_check(want, got):
    want = np.asarray(want, np.float64)
    got = np.asarray(got, np.float64)
    assert want.shape == got.shape
    tol = max(FIXTURE_TOL, FIXTURE_TOL * np.abs(want).max())
    assert np.abs(want - got).max() <= tol
    assert cosine(want, got) > 0.999999


@pytest.mark.parametrize("case", ["matmulnbits_basic", "matmulnbits_zeropoints",
                                  "matmulnbits_partial_block"])
def test_oracle_matmulnbits_fixtures(golden, case):
    g = golden(case)
    a = g["meta"]["attrs"]
    zp = g.get("init_z")
    y = O.matmul_nbits(g["in_a"], g["init_b"], g["init_s"], zp, a["K"], a["N"], a["bits"],
                       a["block_size"])
    _fixture_check(g["expected"], y)


def test_oracle_gemm_fixture(golden):
    g = golden("gemm_transB_bias")
    at = g["meta"]["attrs"]
    y = O.gemm(g["in_x"], g["init_w"], g["init_c"], alpha=at["alpha"], beta=at["beta"],
               transB=bool(at["transB"]))
    _fixture_check(g["expected"], y)


def test_oracle_matmul_batched_fixture(golden):
    g = golden("matmul_batched")
    _fixture_check(g["expected"], O.matmul(g["in_a"], g["in_b"]))


def test_oracle_gemm_prepack_known_answer():
    # test/gemm_prepack_test.dart:113-156: X [2,3] . W^T (W [4,3]) + C.
    w = np.arange(1, 13, dtype=np.float32).reshape(4, 3)
    x = np.arange(1, 7, dtype=np.float32).reshape(2, 3)
    c = np.array([10, 20, 30, 40], np.float32)
    y = O.gemm(x, w, c, transB=True)
    assert y.ravel().tolist() == [24.0, 52.0, 80.0, 108.0, 42.0, 97.0, 152.0, 207.0]


def test_half_to_float_known_values():
    # test/loader_test.dart:78-87
    v = O.half_to_float(np.array([0x0000, 0x3C00, 0xC000, 0x3555], np.uint16))
    assert v[0] == 0.0 and v[1] == 1.0 and v[2] == -2.0
    assert abs(v[3] - 0.333) < 1e-3


def test_half_to_float_all_patterns_bit_exact():
    h = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    got = O.half_to_float(h).view(np.uint32)
    want = h.view(np.float16).astype(np.float32).view(np.uint32)
    nan = np.isnan(h.view(np.float16))
    assert np.array_equal(got[~nan], want[~nan])
    # NaN payloads: sign | 0x7F800000 | mant << 13 (onnx_proto_loader.dart:43)
    hn = h[nan].astype(np.uint32)
    assert np.array_equal(got[nan], ((hn & 0x8000) << 16) | 0x7F800000 | ((hn & 0x3FF) << 13))


def _naive(a, b):
    return (a.astype(np.float64) @ b.astype(np.float64)).astype(np.float32)


def test_oracle_kernel_exhaustive_small():
    # test/gemm_kernel_test.dart:45-60
    rng = np.random.default_rng(11)
    for m in range(1, 7):
        for k in range(1, 7):
            for n in range(1, 7):
                a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
                b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
                assert np.abs(O.matmul_kernel(a, b) - _naive(a, b)).max() < 1e-5


@pytest.mark.parametrize("m,k,n", [(1, 384, 384), (33, 65, 17), (7, 128, 5), (128, 64, 128),
                                   (5, 1, 9), (64, 384, 1), (1, 40, 151), (1, 128, 19),
                                   (1, 896, 512)])
def test_oracle_kernel_shapes(m, k, n):
    # test/gemm_kernel_test.dart:62-78
    rng = np.random.default_rng(m * 1000 + k + n)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    assert np.abs(O.matmul_kernel(a, b) - _naive(a, b)).max() < 1e-4


def test_oracle_fp32_order_matches_definition():
    # matmulKernel's fp32 columns: c = fl(c + fl(a*b)) ascending k.
    rng = np.random.default_rng(3)
    a = rng.standard_normal((3, 50)).astype(np.float32)
    b = rng.standard_normal((50, 8)).astype(np.float32)
    want = np.zeros((3, 8), np.float32)
    for kk in range(50):
        want = (want + (a[:, kk:kk + 1] * b[kk:kk + 1, :]).astype(np.float32)).astype(np.float32)
    assert np.array_equal(O.matmul_kernel(a, b), want)


def test_oracle_gemv_tail_columns_double():
    # m == 1, n % 4 == 3: the last 3 columns accumulate in double
    # (gemm_kernel_simd.dart:299-307), the rest in fp32.
    rng = np.random.default_rng(5)
    k, n = 300, 11
    a = rng.standard_normal((1, k)).astype(np.float32)
    b = rng.standard_normal((k, n)).astype(np.float32)
    y = O.matmul_kernel(a, b)
    acc32 = np.zeros(n, np.float32)
    for kk in range(k):
        acc32 = (acc32 + (a[0, kk] * b[kk]).astype(np.float32)).astype(np.float32)
    acc64 = np.zeros(n, np.float64)
    for kk in range(k):
        acc64 = acc64 + np.float64(a[0, kk]) * b[kk].astype(np.float64)
    assert np.array_equal(y[0, :8], acc32[:8])
    assert np.array_equal(y[0, 8:], acc64[8:].astype(np.float32))


@pytest.mark.parametrize("threads", [2, 3, 7])
def test_oracle_column_split_bitwise(threads):
    # parallel_pool_test.dart: the column-split pool equals the
    # single-threaded result bit for bit.
    rng = np.random.default_rng(23)
    K, N, bs = 256, 150, 32
    B, s, z = O.make_nbits_weight(rng, K, N, bs, zero_points=True)
    for M in (1, 5):
        A = rng.standard_normal((M, K)).astype(np.float32)
        y1 = O.matmul_nbits(A, B, s, z, K, N, 4, bs, threads=1)
        yt = O.matmul_nbits(A, B, s, z, K, N, 4, bs, threads=threads)
        assert np.array_equal(y1, yt)


def test_oracle_dequant_definition():
    rng = np.random.default_rng(9)
    K, N, bs = 40, 5, 32  # partial last block
    B, s, z = O.make_nbits_weight(rng, K, N, bs, zero_points=True)
    W = O.dequant_nbits(B, s, z, K, N, bs)
    nb = 2
    for n in range(N):
        for k in range(K):
            blk, j = divmod(k, bs)
            byte = B[n, blk, j >> 1]
            q = (byte & 0xF) if j % 2 == 0 else (byte >> 4)
            zi = n * nb + blk
            zv = (z[zi >> 1] & 0xF) if zi % 2 == 0 else (z[zi >> 1] >> 4)
            assert W[k, n] == np.float32((np.float64(q) - zv) * np.float64(s[n * nb + blk]))


def test_oracle_rejects_bits8():
    with pytest.raises(NotImplementedError):
        O.matmul_nbits(np.zeros((1, 32), np.float32), np.zeros((1, 1, 16), np.uint8),
                       np.ones(1, np.float32), None, 32, 1, 8, 32)


def _argminmax_fixture(golden, case):
    g = golden(case)
    meta = g["meta"]
    a = meta["attrs"]
    return g, dict(axis=int(a.get("axis", 0)), keepdims=bool(a.get("keepdims", 1)),
                   is_max=meta["op_type"] == "ArgMax",
                   select_last=bool(a.get("select_last_index", 0)))


@pytest.mark.parametrize("case", ["argmax_axis1", "argmax_nan", "argmin_nokeep_last"])
def test_oracle_argminmax_fixtures(golden, case):
    """ArgMax / ArgMin restatement against the reference's ORT fixtures
    (ties to the first or, with select_last_index, last index; a NaN wins
    only as the first element).  Integer output: exact."""
    g, kw = _argminmax_fixture(golden, case)
    got = O.argminmax(g["in_x"], **kw)
    assert got.dtype == np.int64
    assert np.array_equal(got, g["expected"])


@pytest.mark.parametrize("case", ["matmulinteger_nozp", "matmulinteger_percol_bzp",
                                  "matmulinteger_u8i8", "matmulinteger_batched"])
def test_oracle_matmul_integer_fixtures(golden, case):
    """MatMulInteger restatement against the reference's ORT fixtures:
    exact integers."""
    g = golden(case)
    got = O.matmul_integer(g["init_a"], g["init_b"], g.get("init_az"), g.get("init_bz"))
    assert np.array_equal(got, g["expected"])


def test_oracle_dynamic_quantize_linear_fixture(golden):
    g = golden("dynamicquantizelinear")
    y, scale, zp = O.dynamic_quantize_linear(g["in_x"])
    assert np.array_equal(y.astype(np.int64), g["expected_out0"])
    assert np.float32(scale) == np.float32(g["expected_out1"])
    assert zp == int(g["expected_out2"])


def test_oracle_matmul_integer_float64_is_exact():
    """The float64 form of the MatMulInteger oracle equals exact int64
    arithmetic at an LLM-sized K with extreme operands."""
    rng = np.random.default_rng(4)
    K = 14336
    a = rng.integers(0, 256, (3, K)).astype(np.uint8)
    b = rng.integers(-128, 128, (K, 5)).astype(np.int8)
    a[0] = 255
    b[:, 0] = -128
    az, bz = np.array([0], np.uint8), np.array([127], np.int8)
    want = (a.astype(np.int64) - 0) @ (b.astype(np.int64) - 127)
    assert np.array_equal(O.matmul_integer(a, b, az, bz), want)


@pytest.mark.parametrize("case", ["gqa_causal", "gqa_kvcache", "gqa_kvcache_bias",
                                  "gqa_kvcache_rotary"])
def test_oracle_group_query_attention_fixtures(golden, case):
    """GroupQueryAttention restatement (causal, KV cache, additive bias,
    RoPE) against the reference's ORT fixtures: output and present K/V."""
    from tests.attn_fixtures import gqa_args
    g = golden(case)
    q, k, v, kw = gqa_args(g)
    out, pk, pv = O.group_query_attention(q, k, v, **kw)
    _fixture_check(g["expected_out0"], out)
    outs = [key for key in g if key.startswith("expected_") and key != "expected_out0"]
    if len(outs) == 2:
        _fixture_check(g[sorted(outs)[0]], pk)
        _fixture_check(g[sorted(outs)[1]], pv)


@pytest.mark.parametrize("case", ["mha_no_bias", "mha_with_bias"])
def test_oracle_multi_head_attention_fixtures(golden, case):
    from tests.attn_fixtures import mha_args
    g = golden(case)
    q, k, v, kw = mha_args(g)
    _fixture_check(g["expected"], O.multi_head_attention(q, k, v, **kw))


def test_oracle_rotary_embedding_fixture(golden):
    from tests.attn_fixtures import rotary_args
    g = golden("rotary_embedding")
    args, kw = rotary_args(g)
    _fixture_check(g["expected"], O.rotary_embedding(*args, **kw))


def test_oracle_fused_sdpa_fixture(golden):
    """The MatMul/Div/Add/Softmax/MatMul pattern as the reference fuses it
    (scale = float32(1/c), mask broadcast over heads and rows)."""
    from tests.attn_fixtures import sdpa_args
    g = golden("sdpa_pattern")
    a, b, v, mask, scale = sdpa_args(g)
    _fixture_check(g["expected"], O.fused_sdpa(a, b, v, mask, scale))


def test_oracle_gqa_present_is_past_then_current():
    """present K/V = past followed by the step's (roped) K and raw V, and a
    decode step over the present cache equals the last row of the same
    sequence run as one prefill (the causal mask makes them the same
    computation)."""
    rng = np.random.default_rng(3)
    H, Hkv, D, S = 4, 2, 8, 6
    q = rng.standard_normal((1, S, H * D)).astype(np.float32)
    k = rng.standard_normal((1, S, Hkv * D)).astype(np.float32)
    v = rng.standard_normal((1, S, Hkv * D)).astype(np.float32)
    cos = rng.standard_normal((16, D // 2)).astype(np.float32)
    sin = rng.standard_normal((16, D // 2)).astype(np.float32)
    full, pk, pv = O.group_query_attention(q, k, v, H, Hkv, do_rotary=True, cos_cache=cos,
                                           sin_cache=sin)
    part, pk1, pv1 = O.group_query_attention(q[:, :S - 1], k[:, :S - 1], v[:, :S - 1], H, Hkv,
                                             do_rotary=True, cos_cache=cos, sin_cache=sin)
    step, pk2, pv2 = O.group_query_attention(q[:, S - 1:], k[:, S - 1:], v[:, S - 1:], H, Hkv,
                                             do_rotary=True, cos_cache=cos, sin_cache=sin,
                                             past_key=pk1, past_value=pv1)
    assert np.array_equal(pk2, pk) and np.array_equal(pv2, pv)
    assert np.allclose(step[0, 0], full[0, S - 1], rtol=1e-6, atol=1e-6)
    assert np.allclose(part, full[:, :S - 1], rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("case", ["topk_largest", "topk_smallest_axis0"])
def test_oracle_topk_fixtures(golden, case):
    """TopK restatement against the reference's ORT fixtures: values and
    int64 indices exactly."""
    g = golden(case)
    a = g["meta"]["attrs"]
    vals, idx = O.topk(g["in_x"], int(g["init_k"].ravel()[0]), axis=int(a.get("axis", -1)),
                       largest=bool(a.get("largest", 1)))
    assert np.array_equal(vals, g["expected_out0"])
    assert np.array_equal(idx, g["expected_out1"])


def test_oracle_topk_ties_nan_and_signed_zero():
    """Ties keep index order, NaN ranks above every number (first when
    largest, last when smallest), -0.0 ties with 0.0."""
    x = np.array([[1.0, np.nan, 3.0, 3.0, -0.0, 0.0, np.inf, -np.inf]], np.float32)
    v, i = O.topk(x, 8)
    assert i.tolist() == [[1, 6, 2, 3, 0, 4, 5, 7]]
    v, i = O.topk(x, 8, largest=False)
    assert i.tolist() == [[7, 4, 5, 0, 2, 3, 6, 1]]
    assert np.array_equal(O.slice_last_seq(np.arange(24.0).reshape(2, 3, 4)),
                          np.arange(24.0).reshape(2, 3, 4)[:, 2:3])
