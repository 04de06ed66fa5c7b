"""Device attention of a decoder step (ort_cuda_group_query_attention,
ort_cuda_multi_head_attention, ort_cuda_fused_sdpa,
ort_cuda_rotary_embedding) against the oracle's restatements of
opGroupQueryAttention / opMultiHeadAttention / opFusedSDPA /
opRotaryEmbedding (lib/src/onnx_ops.dart:1507-1774, :2121-2172), which are
pinned to the reference's ORT fixtures (tests/test_oracle.py).

Tolerance: exact mode, max|dY| / max|Y_ref| <= 1e-5 (fp32 FMA dot products
and expf instead of the reference's separately rounded products and double
exp); the reference fixtures themselves at their own 2e-5.  RoPE and the
present K/V cache are bit-exact (the same double arithmetic, stored fp32;
the cache is a copy).
"""
import numpy as np
import pytest

from oracle import oracle as O
from tests.attn_fixtures import GQA_CASES, MHA_CASES, gqa_args, mha_args, rotary_args, sdpa_args
from tests.conftest import max_rel

pytestmark = pytest.mark.gpu
TOL = 1e-5
FIXTURE_TOL = 2e-5


@pytest.fixture(scope="module")
def sess():
    from onnx_runtime_dart_b200 import CudaSession
    s = CudaSession(0)
    yield s
    s.close()


def _fixture_ok(want, got):
    want = np.asarray(want, np.float64)
    got = np.asarray(got, np.float64)
    assert want.shape == got.shape
    assert np.abs(want - got).max() <= max(FIXTURE_TOL, FIXTURE_TOL * np.abs(want).max())


@pytest.mark.parametrize("case", GQA_CASES)
def test_gqa_reference_fixtures(sess, golden, case):
    g = golden(case)
    q, k, v, kw = gqa_args(g)
    out, pk, pv = sess.group_query_attention(q, k, v, **kw)
    _fixture_ok(g["expected_out0"], out)
    want_o, want_k, want_v = O.group_query_attention(q, k, v, **kw)
    assert max_rel(want_o, out) <= TOL
    assert np.array_equal(pk, want_k) and np.array_equal(pv, want_v)


@pytest.mark.parametrize("case", MHA_CASES)
def test_mha_reference_fixtures(sess, golden, case):
    g = golden(case)
    q, k, v, kw = mha_args(g)
    out = sess.multi_head_attention(q, k, v, **kw)
    _fixture_ok(g["expected"], out)
    assert max_rel(O.multi_head_attention(q, k, v, **kw), out) <= TOL


def test_rotary_reference_fixture(sess, golden):
    g = golden("rotary_embedding")
    args, kw = rotary_args(g)
    y = sess.rotary_embedding(*args, **kw)
    _fixture_ok(g["expected"], y)
    assert np.array_equal(y, O.rotary_embedding(*args, **kw))


def test_sdpa_reference_fixture(sess, golden):
    g = golden("sdpa_pattern")
    a, b, v, mask, scale = sdpa_args(g)
    out = sess.fused_sdpa(a, b, v, mask, scale)
    _fixture_ok(g["expected"], out)
    assert max_rel(O.fused_sdpa(a, b, v, mask, scale), out) <= TOL


def _gqa_inputs(rng, B, S, P, H, Hkv, D, rotary=False, bias=False, max_pos=None):
    q = rng.standard_normal((B, S, H * D)).astype(np.float32)
    k = rng.standard_normal((B, S, Hkv * D)).astype(np.float32)
    v = rng.standard_normal((B, S, Hkv * D)).astype(np.float32)
    kw = dict(num_heads=H, kv_num_heads=Hkv)
    if P:
        kw["past_key"] = rng.standard_normal((B, Hkv, P, D)).astype(np.float32)
        kw["past_value"] = rng.standard_normal((B, Hkv, P, D)).astype(np.float32)
    if rotary:
        mp = max_pos or P + S + 3
        ang = rng.uniform(0, 6.3, (mp, D // 2))
        kw.update(do_rotary=True, cos_cache=np.cos(ang).astype(np.float32),
                  sin_cache=np.sin(ang).astype(np.float32))
    if bias:
        kw["attention_bias"] = (rng.standard_normal((B, 2, S, P + S)) * 0.5).astype(np.float32)
    return q, k, v, kw


# (batch, seq, past, heads, kv heads, head size): decode (1 query token over
# a long past: split keys), GQA groups of 1/4/8, prefill tiles of 64 rows
# with ragged edges, head sizes 8/64/80/128
GQA_SHAPES = [
    (1, 1, 0, 4, 2, 8),
    (1, 1, 300, 32, 8, 64),
    (4, 1, 639, 32, 8, 64),
    (2, 1, 1000, 32, 8, 128),
    (3, 2, 77, 8, 8, 64),
    (1, 5, 3, 4, 2, 16),
    (2, 37, 0, 8, 2, 64),
    (1, 70, 20, 16, 2, 128),
    (2, 33, 5, 6, 3, 80),
]


@pytest.mark.parametrize("shape", GQA_SHAPES)
@pytest.mark.parametrize("rotary,bias", [(False, False), (True, False), (True, True)])
def test_gqa_matches_oracle(sess, shape, rotary, bias):
    B, S, P, H, Hkv, D = shape
    rng = np.random.default_rng(hash(shape) % 2 ** 32)
    q, k, v, kw = _gqa_inputs(rng, B, S, P, H, Hkv, D, rotary, bias)
    want_o, want_k, want_v = O.group_query_attention(q, k, v, **kw)
    out, pk, pv = sess.group_query_attention(q, k, v, **kw)
    assert max_rel(want_o, out) <= TOL, max_rel(want_o, out)
    assert np.array_equal(pk, want_k) and np.array_equal(pv, want_v)
    # the same call again: split-key tickets are back at zero
    out2, _, _ = sess.group_query_attention(q, k, v, **kw)
    assert np.array_equal(out, out2)


def test_gqa_interleaved_rotary_and_scale(sess):
    rng = np.random.default_rng(11)
    q, k, v, kw = _gqa_inputs(rng, 2, 3, 9, 8, 4, 32, rotary=True)
    kw.update(rotary_interleaved=True, scale=0.3)
    want_o, want_k, _ = O.group_query_attention(q, k, v, **kw)
    out, pk, _ = sess.group_query_attention(q, k, v, **kw)
    assert max_rel(want_o, out) <= TOL
    assert np.array_equal(pk, want_k)


def test_gqa_device_decode_loop_in_place_cache(sess):
    """Prefill, then decode steps on torch device tensors with an in-place
    KV cache of fixed capacity (present = past buffer): every step equals
    the oracle run with the dense past of the previous step."""
    import torch
    rng = np.random.default_rng(5)
    B, H, Hkv, D, S0, steps, cap = 2, 8, 2, 64, 19, 6, 64
    ang = rng.uniform(0, 6.3, (cap, D // 2))
    cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    kc = torch.zeros((B, Hkv, cap, D), device="cuda")
    vc = torch.zeros_like(kc)
    tc, ts = torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda()
    past_k = past_v = None
    past = 0
    for step in range(steps + 1):
        S = S0 if step == 0 else 1
        q = rng.standard_normal((B, S, H * D)).astype(np.float32)
        k = rng.standard_normal((B, S, Hkv * D)).astype(np.float32)
        v = rng.standard_normal((B, S, Hkv * D)).astype(np.float32)
        want_o, past_k, past_v = O.group_query_attention(
            q, k, v, H, Hkv, do_rotary=True, cos_cache=cos, sin_cache=sin,
            past_key=past_k, past_value=past_v)
        out, _, _ = sess.group_query_attention(
            torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(),
            H, Hkv, do_rotary=True, cos_cache=tc, sin_cache=ts, past_key=kc, past_value=vc,
            past_len=past, present_key=kc, present_value=vc)
        torch.cuda.synchronize()
        assert max_rel(want_o, out.cpu().numpy()) <= TOL
        past += S
        assert np.array_equal(kc[:, :, :past].cpu().numpy(), past_k)
        assert np.array_equal(vc[:, :, :past].cpu().numpy(), past_v)


@pytest.mark.parametrize("B,S,KV,H,hidden", [(1, 5, 5, 4, 24), (2, 17, 40, 4, 256),
                                             (3, 1, 700, 8, 512), (1, 100, 130, 2, 128)])
@pytest.mark.parametrize("bias", [False, True])
def test_mha_matches_oracle(sess, B, S, KV, H, hidden, bias):
    rng = np.random.default_rng(B * 1000 + S)
    q = rng.standard_normal((B, S, hidden)).astype(np.float32)
    k = rng.standard_normal((B, KV, hidden)).astype(np.float32)
    v = rng.standard_normal((B, KV, hidden)).astype(np.float32)
    ab = (rng.standard_normal((1, H, S, KV)) * 0.5).astype(np.float32) if bias else None
    want = O.multi_head_attention(q, k, v, H, attention_bias=ab)
    got = sess.multi_head_attention(q, k, v, H, attention_bias=ab)
    assert max_rel(want, got) <= TOL


@pytest.mark.parametrize("lead,S,T,D,Dv,mshape", [
    ((2, 3), 4, 4, 8, 8, (2, 1, 1, 4)),
    ((1, 8), 64, 64, 64, 64, (1, 1, 64, 64)),
    ((2, 4), 1, 300, 64, 32, (2, 4, 1, 300)),
    ((6,), 33, 50, 6, 10, (50,)),
])
def test_sdpa_matches_oracle(sess, lead, S, T, D, Dv, mshape):
    rng = np.random.default_rng(S * 7 + T)
    a = rng.standard_normal(lead + (S, D)).astype(np.float32)
    b = rng.standard_normal(lead + (D, T)).astype(np.float32)
    v = rng.standard_normal(lead + (T, Dv)).astype(np.float32)
    mask = np.where(rng.random(mshape) < 0.2, -1e4, 0.0).astype(np.float32)
    scale = float(np.float32(1 / np.sqrt(D)))
    want = O.fused_sdpa(a, b, v, mask, scale)
    assert max_rel(want, sess.fused_sdpa(a, b, v, mask, scale)) <= TOL


@pytest.mark.parametrize("x_shape,nh,interleaved,rdim", [((2, 7, 96), 4, False, 0),
                                                        ((2, 7, 96), 4, True, 0),
                                                        ((1, 3, 5, 32), 0, False, 16),
                                                        ((2, 9, 64), 2, False, 20)])
def test_rotary_matches_oracle_bitwise(sess, x_shape, nh, interleaved, rdim):
    rng = np.random.default_rng(len(x_shape) * 10 + nh)
    x = rng.standard_normal(x_shape).astype(np.float32)
    seq = x_shape[2] if len(x_shape) == 4 else x_shape[1]
    half = 16 if len(x_shape) == 4 else (x_shape[2] // nh) // 2
    ang = rng.uniform(0, 6.3, (40, half))
    cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    pos = rng.integers(0, 40, (x_shape[0], seq)).astype(np.int64)
    want = O.rotary_embedding(x, pos, cos, sin, interleaved, nh, rdim)
    got = sess.rotary_embedding(x, pos, cos, sin, interleaved, nh, rdim)
    assert np.array_equal(want, got)


def test_attention_rejects_bad_arguments(sess):
    from onnx_runtime_dart_b200 import UnsupportedError
    rng = np.random.default_rng(0)
    q = rng.standard_normal((1, 2, 2 * 256)).astype(np.float32)
    kv = rng.standard_normal((1, 2, 256)).astype(np.float32)
    with pytest.raises(UnsupportedError):
        sess.group_query_attention(q, kv, kv, 2, 1)
    q = rng.standard_normal((1, 2, 3 * 8)).astype(np.float32)
    kv = rng.standard_normal((1, 2, 2 * 8)).astype(np.float32)
    with pytest.raises(ValueError):
        sess.group_query_attention(q, kv, kv, 3, 2)


@pytest.mark.parametrize("shape", [(2, 1, 200, 8, 2, 64), (1, 40, 9, 8, 4, 64)])
@pytest.mark.parametrize("interleaved", [False, True])
def test_gqa_partial_rotary(sess, shape, interleaved):
    """cos/sin caches of head/4 values: RoPE on the first head/2 features of
    Q and K, the rest passed through (decode kernel and prefill pre-pass)."""
    B, S, P, H, Hkv, D = shape
    rng = np.random.default_rng(21)
    q, k, v, kw = _gqa_inputs(rng, B, S, P, H, Hkv, D)
    ang = rng.uniform(0, 6.3, (P + S + 2, D // 4))
    kw.update(do_rotary=True, rotary_interleaved=interleaved,
              cos_cache=np.cos(ang).astype(np.float32), sin_cache=np.sin(ang).astype(np.float32))
    want_o, want_k, want_v = O.group_query_attention(q, k, v, **kw)
    out, pk, pv = sess.group_query_attention(q, k, v, **kw)
    assert max_rel(want_o, out) <= TOL
    assert np.array_equal(pk, want_k) and np.array_equal(pv, want_v)


@pytest.mark.parametrize("case", GQA_CASES + MHA_CASES + ["rotary_embedding"])
def test_dispatch_attention_fixture_nodes(sess, golden, case):
    """The fixture's node through CudaSession.dispatch, as the reference's
    OnnxGraphExecutor._dispatch would route it (onnx_graph.dart:978-1005):
    every output against the ORT-computed fixture."""
    g = golden(case)
    node = g["meta"]
    values = {k[3:]: v for k, v in g.items() if k.startswith("in_")}
    values.update({k[5:]: v for k, v in g.items() if k.startswith("init_")})
    outs = sess.dispatch(node, values)
    names = sorted(k for k in g if k.startswith("expected_"))
    for name, got in zip(names, outs):
        _fixture_ok(g[name], np.asarray(got))
