"""GPU parity: the CUDA path (through the C ABI) against the CPU oracle and
the reference's fixtures.

Tolerances (from the task's stated parity bar):
  exact mode   max|dY| / max|Y_ref| <= 1e-5
  strict mode  bitwise equal to the oracle (the reference's rounding)
  fixtures     the reference's own bar: max|dY| <= max(2e-5, 2e-5*max|Y|)
               and cosine > 0.999999 (fixture_parity_test.dart:21,242,256)
"""
import numpy as np
import pytest

from oracle import oracle as O
from tests.conftest import cosine, max_rel

pytestmark = pytest.mark.gpu

EXACT_TOL = 1e-5


@pytest.fixture(scope="module")
def sess():
    from onnx_runtime_dart_b200 import CudaSession
    s = CudaSession(0, mode="exact")
    yield s
    s.close()


def _flags(mode):
    from onnx_runtime_dart_b200 import _lib
    return _lib.flags_mode(_lib.MODES[mode])


def _fixture_ok(want, got):
    want = np.asarray(want, np.float64)
    assert want.shape == got.shape
    tol = max(2e-5, 2e-5 * np.abs(want).max())
    assert np.abs(want - got).max() <= tol
    assert cosine(want, got) > 0.999999


# ---- the reference's fixtures ------------------------------------------------

@pytest.mark.parametrize("case", ["matmulnbits_basic", "matmulnbits_zeropoints",
                                  "matmulnbits_partial_block"])
@pytest.mark.parametrize("mode", ["exact", "strict"])
def test_fixture_matmulnbits(sess, golden, case, mode):
    g = golden(case)
    at = g["meta"]["attrs"]
    zp = g.get("init_z")
    sess.upload_nbits("fx", g["init_b"], g["init_s"], zp, k=at["K"], n=at["N"],
                      bits=at["bits"], block_size=at["block_size"])
    y = sess.matmul_nbits("fx", g["in_a"], flags=_flags(mode))
    _fixture_ok(g["expected"], y)
    ref = O.matmul_nbits(g["in_a"], g["init_b"], g["init_s"], zp, at["K"], at["N"], 4,
                         at["block_size"])
    if mode == "strict":
        assert np.array_equal(y, ref)
    else:
        assert max_rel(ref, y) <= EXACT_TOL


@pytest.mark.parametrize("mode", ["exact", "strict"])
def test_fixture_gemm(sess, golden, mode):
    g = golden("gemm_transB_bias")
    at = g["meta"]["attrs"]
    sess.upload_dense("w", g["init_w"], trans_b=bool(at["transB"]))
    y = sess.gemm("w", g["in_x"], g["init_c"], alpha=at["alpha"], beta=at["beta"],
                  flags=_flags(mode))
    _fixture_ok(g["expected"], y)
    ref = O.gemm(g["in_x"], g["init_w"], g["init_c"], transB=True)
    if mode == "strict":
        assert np.array_equal(y, ref)


@pytest.mark.parametrize("mode", ["exact", "strict"])
def test_fixture_matmul_batched(sess, golden, mode):
    g = golden("matmul_batched")
    y = sess.matmul_batched(g["in_a"], g["in_b"], flags=_flags(mode))
    _fixture_ok(g["expected"], y)
    if mode == "strict":
        assert np.array_equal(y, O.matmul(g["in_a"], g["in_b"]))


def test_gemm_prepack_known_answer_twice(sess):
    # test/gemm_prepack_test.dart:113-156 (second run uses the resident copy)
    w = np.arange(1, 13, dtype=np.float32).reshape(4, 3)
    x = np.arange(1, 7, dtype=np.float32).reshape(2, 3)
    c = np.array([10, 20, 30, 40], np.float32)
    sess.upload_dense("W", w, trans_b=True)
    want = [24.0, 52.0, 80.0, 108.0, 42.0, 97.0, 152.0, 207.0]
    for _ in range(2):
        for mode in ("exact", "strict"):
            assert sess.gemm("W", x, c, flags=_flags(mode)).ravel().tolist() == want


# ---- MatMulNBits at the benchmark configurations ----------------------------

def _nbits_case(sess, rng, M, K, N, bs, zp, scale_dtype=np.float32, mode="exact",
                threads=8, name="w"):
    B, s, z = O.make_nbits_weight(rng, K, N, bs, zero_points=zp, scale_dtype=scale_dtype)
    A = rng.standard_normal((M, K)).astype(np.float32)
    sess.upload_nbits(name, B, s, z, k=K, n=N, block_size=bs)
    y = sess.matmul_nbits(name, A, flags=_flags(mode))
    s32 = s.astype(np.float32) if scale_dtype == np.float16 else s
    ref = O.matmul_nbits(A, B, s32, z, K, N, 4, bs, threads=threads)
    return ref, y


def test_cfg1_single_op(sess):
    # A [1,16,1024], K=N=1024, bs 32, no zp, seed 0
    rng = np.random.default_rng(0)
    ref, y = _nbits_case(sess, rng, 16, 1024, 1024, 32, False)
    assert max_rel(ref, y) <= EXACT_TOL


QWEN3_PROJ = [(1024, 2048), (1024, 1024), (2048, 1024), (1024, 3072), (3072, 1024),
              (1024, 151936)]


@pytest.mark.parametrize("K,N", QWEN3_PROJ)
def test_cfg3_decode_projections(sess, K, N):
    # M=1, bs 32, fp32 scales, packed zero points
    rng = np.random.default_rng(K * 7 + N)
    ref, y = _nbits_case(sess, rng, 1, K, N, 32, True)
    assert max_rel(ref, y) <= EXACT_TOL


@pytest.mark.parametrize("M", [1, 2, 3, 4, 5, 8, 16, 33])
@pytest.mark.parametrize("zp", [False, True])
def test_gemv_and_tiled_rows(sess, M, zp):
    rng = np.random.default_rng(100 + M + 7 * zp)
    ref, y = _nbits_case(sess, rng, M, 2048, 520, 128, zp, scale_dtype=np.float16)
    assert max_rel(ref, y) <= EXACT_TOL


@pytest.mark.parametrize("bs", [16, 32, 64, 128, 256])
@pytest.mark.parametrize("M", [1, 3, 7])
def test_block_sizes(sess, bs, M):
    rng = np.random.default_rng(bs + M)
    ref, y = _nbits_case(sess, rng, M, 1024 + 512, 77, bs, True)
    assert max_rel(ref, y) <= EXACT_TOL


@pytest.mark.parametrize("K", [16, 40, 48, 80, 1000, 1040, 3104])
def test_ragged_k(sess, K):
    # partial last blocks and K not a multiple of the 1024-k warp step
    rng = np.random.default_rng(K)
    for M in (1, 2, 6):
        ref, y = _nbits_case(sess, rng, M, K, 37, 32 if K % 32 == 0 else 16, True)
        assert max_rel(ref, y) <= EXACT_TOL


@pytest.mark.parametrize("M,K,N,bs", [(1, 64, 8, 32), (1, 40, 151, 32), (1, 128, 19, 16),
                                      (3, 96, 10, 32), (4, 256, 130, 64), (9, 80, 5, 16)])
def test_strict_bitwise(sess, M, K, N, bs):
    # strict mode reproduces the reference's rounding exactly, including
    # the double-accumulated m == 1 tail columns (n % 4 != 0)
    rng = np.random.default_rng(M * K + N)
    ref, y = _nbits_case(sess, rng, M, K, N, bs, True, mode="strict")
    assert np.array_equal(ref, y)


def test_zero_point_layouts_agree_for_even_nb(sess):
    rng = np.random.default_rng(4)
    K, N, bs = 256, 12, 32  # nb = 8 (even): flat == per-column
    B, s, z = O.make_nbits_weight(rng, K, N, bs, zero_points=True)
    A = rng.standard_normal((2, K)).astype(np.float32)
    sess.upload_nbits("flat", B, s, z, k=K, n=N, block_size=bs)
    sess.upload_nbits("col", B, s, z, k=K, n=N, block_size=bs, zp_per_column=True)
    assert np.array_equal(sess.matmul_nbits("flat", A), sess.matmul_nbits("col", A))


def test_zero_point_per_column_odd_nb(sess):
    # ORT spec layout: ceil(nb/2) bytes per column.  Compare against the
    # oracle fed the equivalent flat layout.
    rng = np.random.default_rng(5)
    K, N, bs = 96, 7, 32  # nb = 3
    nb = 3
    B, s, _ = O.make_nbits_weight(rng, K, N, bs, zero_points=False)
    zv = rng.integers(0, 16, size=(N, nb), dtype=np.uint8)
    per_col = np.zeros((N, 2), np.uint8)
    per_col[:, 0] = zv[:, 0] | (zv[:, 1] << 4)
    per_col[:, 1] = zv[:, 2]
    flat = O.pack_nibbles(np.concatenate([zv.ravel(), np.zeros(1, np.uint8)]))
    A = rng.standard_normal((1, K)).astype(np.float32)
    sess.upload_nbits("pc", B, s, per_col, k=K, n=N, block_size=bs, zp_per_column=True)
    ref = O.matmul_nbits(A, B, s, flat, K, N, 4, bs)
    assert max_rel(ref, sess.matmul_nbits("pc", A)) <= EXACT_TOL


@pytest.mark.parametrize("M", [3, 4, 5])
@pytest.mark.parametrize("N", [25000, 40000])
def test_single_d_buffer_many_items(sess, M, N):
    """Block size 32 at M = 3..5 needs all of the D columns for one item (a
    single accumulator buffer) and, at these N, each CTA handles several
    items: the two epilogue groups then share that buffer."""
    rng = np.random.default_rng(M * 7 + N)
    ref, y = _nbits_case(sess, rng, M, 1024, N, 32, True)
    assert max_rel(ref, y) <= EXACT_TOL


def test_split_k_repeat_bitwise(sess):
    """Split-K decode GEMVs write chunk partials that a dependent kernel,
    launched to overlap the GEMV's tail, adds in chunk order.  Repeated and
    interleaved calls on two split-K weights sharing the session scratch
    must reproduce their first results bit for bit."""
    rng = np.random.default_rng(21)
    shapes = {"sk1": (4096, 3000, 128, 1), "sk2": (14336, 1024, 128, 4)}
    A, first = {}, {}
    for name, (K, N, bs, M) in shapes.items():
        B, s, z = O.make_nbits_weight(rng, K, N, bs, zero_points=True)
        sess.upload_nbits(name, B, s, z, k=K, n=N, block_size=bs)
        A[name] = rng.standard_normal((M, K)).astype(np.float32)
        first[name] = sess.matmul_nbits(name, A[name])
        ref = O.matmul_nbits(A[name], B, s, z, K, N, 4, bs, threads=8)
        assert max_rel(ref, first[name]) <= EXACT_TOL
    for _ in range(3):
        for name in shapes:
            assert np.array_equal(sess.matmul_nbits(name, A[name]), first[name])


def test_shard_columns_bitwise_invariant(sess):
    """A column's result does not depend on which other columns are computed
    with it -- the property N-sharding relies on (parallel_pool_test.dart's
    bitwise invariant).  Column slices uploaded as separate weights must
    reproduce the full-weight result bit for bit."""
    rng = np.random.default_rng(6)
    K, N, bs = 4096, 1000, 128
    B, s, z = O.make_nbits_weight(rng, K, N, bs, zero_points=True)
    nb = K // bs
    zv = np.stack([z & 0xF, z >> 4], 1).ravel()[:N * nb].reshape(N, nb)
    for M in (1, 4, 20):
        A = rng.standard_normal((M, K)).astype(np.float32)
        sess.upload_nbits("full", B, s, z, k=K, n=N, block_size=bs)
        full = sess.matmul_nbits("full", A)
        for world in (2, 4, 8):
            per = ((N + world - 1) // world + 3) // 4 * 4
            parts = []
            for r in range(world):
                a, b = min(N, r * per), min(N, (r + 1) * per)
                if a == b:
                    continue
                zr = O.pack_nibbles(np.concatenate(
                    [zv[a:b].ravel(), np.zeros(((b - a) * nb) % 2, np.uint8)]))
                sess.upload_nbits("part", B[a:b], s[a * nb:b * nb], zr, k=K, n=b - a,
                                  block_size=bs)
                parts.append(sess.matmul_nbits("part", A))
            assert np.array_equal(np.concatenate(parts, axis=-1), full)


def test_full_size_lm_head_vs_torch(sess):
    """Llama-3-8B lm_head (4096 -> 128256, bs 128, fp16 scales, zp) at full
    size against an fp64 torch reference of the dequantised weight (the
    oracle is too slow at this size)."""
    import torch
    rng = np.random.default_rng(7)
    K, N, bs = 4096, 128256, 128
    B, s, z = O.make_nbits_weight(rng, K, N, bs, zero_points=True, scale_dtype=np.float16)
    A = rng.standard_normal((1, K)).astype(np.float32)
    sess.upload_nbits("lm", B, s, z, k=K, n=N, block_size=bs)
    y = sess.matmul_nbits("lm", A)
    nb = K // bs
    dev = torch.device("cuda")
    Bt = torch.from_numpy(B).to(dev).reshape(N, nb * bs // 2)
    q = torch.stack([Bt & 0xF, Bt >> 4], -1).reshape(N, nb, bs).double()
    zt = torch.from_numpy(z).to(dev)
    zz = torch.stack([zt & 0xF, zt >> 4], -1).reshape(-1)[:N * nb].reshape(N, nb, 1).double()
    st = torch.from_numpy(s.astype(np.float32)).to(dev).reshape(N, nb, 1).double()
    W = ((q - zz) * st).reshape(N, K).float().double()  # reference rounds W to fp32
    ref = (torch.from_numpy(A).to(dev).double() @ W.T).cpu().numpy()
    sess.drop_weight("lm")
    assert max_rel(ref, y) <= EXACT_TOL


# ---- dense fp32 MatMul / Gemm -------------------------------------------------

@pytest.mark.parametrize("M,K,N", [(1024, 384, 1536), (1024, 1536, 384)])
@pytest.mark.parametrize("mode", ["exact", "strict"])
def test_cfg2_bert_ffn(sess, M, K, N, mode):
    # Gemm transB=1 + bias, seed 1
    rng = np.random.default_rng(1)
    A = rng.standard_normal((M, K)).astype(np.float32)
    W = (rng.standard_normal((N, K)) * 0.05).astype(np.float32)
    c = (rng.standard_normal(N) * 0.02).astype(np.float32)
    sess.upload_dense("ffn", W, trans_b=True)
    y = sess.gemm("ffn", A, c, flags=_flags(mode))
    ref = O.gemm(A, W, c, transB=True, threads=8)
    if mode == "strict":
        assert np.array_equal(y, ref)
    else:
        assert max_rel(ref, y) <= EXACT_TOL


@pytest.mark.parametrize("cshape", [None, (), (9,), (1, 9), (6, 9), (6, 1)])
@pytest.mark.parametrize("alpha,beta", [(1.0, 1.0), (2.0, 0.5), (-0.75, 3.0)])
def test_gemm_epilogue_variants(sess, cshape, alpha, beta):
    rng = np.random.default_rng(11)
    A = rng.standard_normal((6, 13)).astype(np.float32)
    W = rng.standard_normal((13, 9)).astype(np.float32)
    C = None if cshape is None else rng.standard_normal(cshape).astype(np.float32)
    sess.upload_dense("g", W, trans_b=False)
    y = sess.gemm("g", A, C, alpha=alpha, beta=beta, flags=_flags("strict"))
    assert np.array_equal(y, O.gemm(A, W, C, alpha=alpha, beta=beta))


def test_gemm_trans_a(sess):
    rng = np.random.default_rng(12)
    At = rng.standard_normal((13, 6)).astype(np.float32)  # [K, M]
    W = rng.standard_normal((9, 13)).astype(np.float32)
    sess.upload_dense("g", W, trans_b=True)
    y = sess.gemm("g", At, None, trans_a=True, flags=_flags("strict"))
    assert np.array_equal(y, O.gemm(At, W, None, transA=True, transB=True))


@pytest.mark.parametrize("m,k,n", [(1, 384, 384), (33, 65, 17), (7, 128, 5), (128, 64, 128),
                                   (5, 1, 9), (64, 384, 1), (1, 40, 151), (1, 128, 19),
                                   (1, 896, 512)])
def test_kernel_shapes_strict(sess, m, k, n):
    # test/gemm_kernel_test.dart:62-78 shapes, bitwise against the oracle
    rng = np.random.default_rng(m + k + n)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    sess.upload_dense("mm", b)
    assert np.array_equal(sess.matmul("mm", a, flags=_flags("strict")), O.matmul_kernel(a, b))
    assert max_rel(O.matmul_kernel(a, b), sess.matmul("mm", a)) <= EXACT_TOL


def test_exhaustive_small_shapes(sess):
    # test/gemm_kernel_test.dart:45-60
    rng = np.random.default_rng(11)
    for m in range(1, 7):
        for k in range(1, 7):
            for n in range(1, 7):
                a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
                b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
                sess.upload_dense("e", b)
                assert np.array_equal(sess.matmul("e", a, flags=_flags("strict")),
                                      O.matmul_kernel(a, b))


# ---- device residency, dispatch and errors --------------------------------------

def test_device_resident_chain(sess):
    """Activations stay on the device between consecutive hot ops."""
    from onnx_runtime_dart_b200 import DeviceTensor
    rng = np.random.default_rng(13)
    K, H, N = 512, 1024, 256
    B1, s1, z1 = O.make_nbits_weight(rng, K, H, 32, zero_points=False)
    B2, s2, z2 = O.make_nbits_weight(rng, H, N, 32, zero_points=True)
    sess.upload_nbits("l1", B1, s1, z1, k=K, n=H, block_size=32)
    sess.upload_nbits("l2", B2, s2, z2, k=H, n=N, block_size=32)
    A = rng.standard_normal((2, K)).astype(np.float32)
    dA = DeviceTensor.from_host(sess, A)
    dH = sess.matmul_nbits("l1", dA)
    dY = sess.matmul_nbits("l2", dH)
    y = dY.numpy()
    h_ref = O.matmul_nbits(A, B1, s1, None, K, H, 4, 32)
    y_ref = O.matmul_nbits(h_ref, B2, s2, z2, H, N, 4, 32)
    assert max_rel(y_ref, y) <= 5 * EXACT_TOL
    for t in (dA, dH, dY):
        t.free()


def test_dispatch_cases(sess, golden):
    g = golden("matmulnbits_zeropoints")
    node = {"op_type": "MatMulNBits", "inputs": ["a", "b", "s", "z"], "attrs": g["meta"]["attrs"]}
    sess.register_initializers([node], {"b": g["init_b"], "s": g["init_s"], "z": g["init_z"]})
    (y,) = sess.dispatch(node, {"a": g["in_a"]})
    _fixture_ok(g["expected"], y)


def test_errors_mirror_reference(sess):
    from onnx_runtime_dart_b200 import UnsupportedError
    with pytest.raises(UnsupportedError):
        sess.upload_nbits("b8", np.zeros((4, 1, 16), np.uint8), np.ones(4, np.float32), None,
                          k=32, n=4, bits=8, block_size=32)
    node = {"op_type": "MatMulNBits", "inputs": ["a", "b", "s", "z", "g_idx"],
            "attrs": {"K": 32, "N": 4, "block_size": 32}}
    with pytest.raises(UnsupportedError):
        sess.dispatch(node, {"a": np.zeros((1, 32), np.float32)})
    with pytest.raises(KeyError):
        sess.matmul_nbits("missing", np.zeros((1, 32), np.float32))
    from onnx_runtime_dart_b200 import _lib
    L = _lib.load()
    a = np.zeros(32, np.float32)
    y = np.zeros(4, np.float32)
    assert L.ort_cuda_matmul_nbits(sess.handle, b"missing", a.ctypes.data, 1, y.ctypes.data,
                                   _lib.HOST_IO) == _lib.ERR_NOT_FOUND
    sess.upload_dense("gw", np.ones((8, 4), np.float32))
    with pytest.raises(ValueError):
        sess.gemm("gw", np.ones((3, 8), np.float32), np.ones((2, 4), np.float32))
    with pytest.raises(ValueError):  # block_size not a power of two
        sess.upload_nbits("bad", np.zeros((4, 1, 12), np.uint8), np.ones(4, np.float32), None,
                          k=24, n=4, block_size=24)


def test_empty_m(sess):
    rng = np.random.default_rng(14)
    B, s, z = O.make_nbits_weight(rng, 64, 8, 32, zero_points=False)
    sess.upload_nbits("e0", B, s, z, k=64, n=8, block_size=32)
    y = sess.matmul_nbits("e0", np.zeros((0, 64), np.float32))
    assert y.shape == (0, 8)


def test_launch_counter_counts_own_kernels(sess):
    rng = np.random.default_rng(15)
    # one 512-k chunk: a single GEMV launch
    B, s, z = O.make_nbits_weight(rng, 512, 256, 32, zero_points=False)
    sess.upload_nbits("lc", B, s, z, k=512, n=256, block_size=32)
    before = sess.launch_count()
    sess.matmul_nbits("lc", rng.standard_normal((1, 512)).astype(np.float32))
    assert sess.launch_count() == before + 1
    # two chunks over two column tiles: split-K, summed either by a cluster
    # of the two chunks' CTAs (one launch) or by a reduction kernel (two)
    B, s, z = O.make_nbits_weight(rng, 1024, 256, 32, zero_points=False)
    sess.upload_nbits("lc2", B, s, z, k=1024, n=256, block_size=32)
    before = sess.launch_count()
    sess.matmul_nbits("lc2", rng.standard_normal((1, 1024)).astype(np.float32))
    assert sess.launch_count() in (before + 1, before + 2)


@pytest.mark.parametrize("K,N,M", [(4096, 128256, 1), (2048, 148 * 3 * 128, 1), (2048, 148 * 3 * 128, 3)])
def test_tile_major_back_to_back(K, N, M):
    """Tile-major decode GEMVs where CTAs own an odd number of tiles, so one
    epilogue group takes two consecutive items at every chunk boundary,
    launched many times back to back on device buffers (each launch
    overlaps its predecessor's tail).  No bounded wait may expire (the
    session reports it at sync) and every result equals the first bit for
    bit and matches the oracle."""
    import torch
    from onnx_runtime_dart_b200 import CudaSession
    s = CudaSession(0, mode="exact")
    try:
        st = torch.cuda.Stream()
        s.set_stream(st.cuda_stream)
        rng = np.random.default_rng(77)
        B, sc, z = O.make_nbits_weight(rng, K, N, 128, zero_points=True)
        s.upload_nbits("w", B, sc, z, k=K, n=N, block_size=128)
        A = rng.standard_normal((M, K)).astype(np.float32)
        reps = 40
        with torch.cuda.stream(st):
            a = torch.from_numpy(A).to("cuda")
            y = torch.empty(reps, M, N, device="cuda")
            for r in range(reps):
                s.matmul_nbits("w", a, out=y[r])
            st.synchronize()
        s.sync()
        out = y.cpu().numpy()
        for r in range(1, reps):
            assert np.array_equal(out[r], out[0]), f"launch {r} differs"
        ref = O.matmul_nbits(A, B, sc, z, K, N, 4, 128, threads=8)
        assert max_rel(ref, out[0]) <= EXACT_TOL
    finally:
        s.close()


def test_opcase_single_op_timer(capsys):
    """The single-op timing utility runs both decode and prefill cases and
    reads the session's error word after its timed launches."""
    import json
    from onnx_runtime_dart_b200 import opcase
    for argv in (["--k", "1024", "--n", "2048", "--m", "1"],
                 ["--k", "1024", "--n", "1024", "--m", "256", "--mode", "mma_f16"],
                 ["--k", "1024", "--n", "2048", "--m", "1", "--graph"]):
        opcase.main(argv + ["--reps", "2", "--warmup", "1"])
        line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
        assert line["us_per_launch"] > 0 and line["m"] == int(argv[5])


@pytest.mark.parametrize("K,N,M,bs,zp", [
    (4096, 6144, 1, 128, True),     # 48 tiles x 8 chunks
    (4096, 4096, 2, 64, False),     # 32 tiles
    (14336, 4096, 1, 128, True),    # 28 chunks over a cluster
    (14336, 512, 3, 32, True),      # 4 tiles, 28 chunks, bs 32
    (4096, 28672, 4, 256, True),    # 224 tiles
    (2560, 3000, 8, 128, False),    # 5 chunks, ragged last tile
    (1536, 16032, 5, 128, True),    # 3 chunks, 126 tiles
])
def test_cluster_plans_parity_and_slice_invariance(sess, K, N, M, bs, zp):
    """Shapes whose plans share tile sets across clusters of 2-8 CTAs (chunk
    ranges per rank, partials summed in the owning CTA's shared memory).
    Results match the oracle, and the first 128 columns uploaded alone (a
    different plan) give the same bits."""
    rng = np.random.default_rng(K * 7 + N + M)
    B, s, z = O.make_nbits_weight(rng, K, N, bs, zero_points=zp)
    A = rng.standard_normal((M, K)).astype(np.float32)
    sess.upload_nbits("cl", B, s, z, k=K, n=N, block_size=bs)
    y = sess.matmul_nbits("cl", A)
    ref = O.matmul_nbits(A, B, s, z, K, N, 4, bs, threads=8)
    assert max_rel(ref, y) <= EXACT_TOL
    nb = K // bs if K % bs == 0 else K // bs + 1
    n1 = 128
    zs = None
    if zp:
        zv = np.stack([z & 0xF, z >> 4], 1).ravel()[:N * nb].reshape(N, nb)[:n1].ravel()
        if zv.size % 2:
            zv = np.append(zv, 0)
        zs = (zv[0::2] | (zv[1::2] << 4)).astype(np.uint8)
    sess.upload_nbits("cl1", B[:n1], s.reshape(N, nb)[:n1].ravel(), zs, k=K, n=n1, block_size=bs)
    y1 = sess.matmul_nbits("cl1", A)
    assert np.array_equal(y1, y[:, :n1])
    sess.drop_weight("cl")
    sess.drop_weight("cl1")


@pytest.mark.parametrize("K,N,M,bs", [(4096, 6144, 1, 128), (14336, 1024, 2, 128),
                                      (1536, 5000, 4, 128), (2048, 512, 4, 128),
                                      (2048, 2048, 5, 32), (2048, 1024, 8, 128),
                                      (1000, 300, 3, 32),
                                      (4096, 777, 5, 256), (3072, 1000, 2, 512)])
def test_every_gemv_plan_gives_the_same_bits(sess, K, N, M, bs):
    """Every candidate decomposition of the decode GEMV (tile-major, the
    cluster sizes that fit, split-K), over block sizes 32-512, ragged K and
    M up to 8, set through ort_cuda_gemv_plan_set,
    gives bit-identical results that match the oracle; plans outside the
    candidate range are refused and -1 restores the automatic choice."""
    rng = np.random.default_rng(K + N + M)
    B, s, z = O.make_nbits_weight(rng, K, N, bs, zero_points=True)
    A = rng.standard_normal((M, K)).astype(np.float32)
    sess.upload_nbits("pl", B, s, z, k=K, n=N, block_size=bs)
    ref = O.matmul_nbits(A, B, s, z, K, N, 4, bs, threads=8)
    first = None
    plan = 0
    while True:
        try:
            sess.set_gemv_plan("pl", M, plan)
        except ValueError:  # ORT_CUDA_ERR_INVALID_ARG: past the last candidate
            break
        assert sess.gemv_plan("pl", M) == plan
        y = sess.matmul_nbits("pl", A)
        if first is None:
            first = y
            assert max_rel(ref, y) <= EXACT_TOL
        assert np.array_equal(y, first), f"plan {plan} differs"
        plan += 1
    assert plan >= 2  # tile-major and at least one other candidate
    sess.set_gemv_plan("pl", M, -1)
    assert sess.gemv_plan("pl", M) == -1
    assert np.array_equal(sess.matmul_nbits("pl", A), first)
    assert sess.gemv_plan("pl", M) >= 0  # timed and chosen on that call
    sess.drop_weight("pl")


@pytest.mark.parametrize("M,bs", [(9, 128), (16, 128), (37, 128), (64, 128), (16, 32), (40, 32)])
def test_decode_rows_beyond_eight_use_row_chunks(sess, M, bs):
    """Decode-sized M above the GEMV's 8 rows (north_star's M <= 16 family,
    cfg1 and cfg5 M=16) runs the exact tensor-core GEMV over row chunks
    (8 rows; 5 for block size 32): each row matches the oracle and equals
    the same row computed alone bit for bit."""
    rng = np.random.default_rng(M * 31 + bs)
    K, N = 2048, 3000
    B, s, z = O.make_nbits_weight(rng, K, N, bs, zero_points=True)
    A = rng.standard_normal((M, K)).astype(np.float32)
    sess.upload_nbits("rc", B, s, z, k=K, n=N, block_size=bs)
    before = sess.launch_count()
    y = sess.matmul_nbits("rc", A)
    chunk = 8 if bs >= 64 else 5
    passes = -(-M // chunk)
    # one GEMV launch per chunk, plus a chunk-sum launch where a plan is split-K
    assert passes <= sess.launch_count() - before <= 2 * passes
    ref = O.matmul_nbits(A, B, s, z, K, N, 4, bs, threads=8)
    assert max_rel(ref, y) <= EXACT_TOL
    for r in (0, M - 1):
        assert np.array_equal(sess.matmul_nbits("rc", A[r:r + 1]), y[r:r + 1])
    sess.drop_weight("rc")
