"""Fused groups of sibling MatMulNBits weights (ort_cuda_fuse_nbits,
ort_cuda_matmul_nbits_group): q/k/v and gate/up, which the reference keeps
as separate nodes on the same input (opMatMulNBits per node,
onnx_graph.dart:1584-1596).  Each part's output must equal, bit for bit,
what ort_cuda_matmul_nbits gives for that part alone, on every path (one
GEMV launch for the group at decode sizes, the whole-op path for STRICT
and prefill sizes, host buffers, CUDA-graph replay); and the parts match the
oracle at the exact mode's bar.
"""
import numpy as np
import pytest

from oracle import oracle as O
from tests.conftest import max_rel

pytestmark = pytest.mark.gpu

K = 2048
PARTS = {"q": 2048, "k": 512, "v": 512}


@pytest.fixture(scope="module")
def grp():
    from onnx_runtime_dart_b200 import CudaSession
    from onnx_runtime_dart_b200.workloads import make_nbits_weight
    rng = np.random.default_rng(44)
    s = CudaSession(0)
    W = {}
    for name, n in PARTS.items():
        W[name] = make_nbits_weight(rng, K, n, 128, zero_points=True, scale_dtype=np.float16)
        s.upload_nbits(name, *W[name], k=K, n=n, block_size=128)
    s.fuse_nbits("qkv", list(PARTS))
    yield s, W
    s.close()


@pytest.mark.parametrize("M", [1, 3, 8, 13])
def test_group_equals_parts(grp, M):
    import torch
    s, W = grp
    a = torch.randn(M, K, device="cuda", generator=torch.Generator("cuda").manual_seed(M))
    before = s.launch_count()
    outs = s.matmul_nbits_group("qkv", a)
    torch.cuda.synchronize()
    group_launches = s.launch_count() - before
    for (name, n), y in zip(PARTS.items(), outs):
        alone = s.matmul_nbits(name, a)
        torch.cuda.synchronize()
        assert torch.equal(y, alone), name
        B, sc, z = W[name]
        ref = O.matmul_nbits(a.cpu().numpy(), B, sc.astype(np.float32), z, K, n, 4, 128,
                             threads=8)
        assert max_rel(ref, y.cpu().numpy()) <= 1e-5
    # one GEMV (+ its chunk sum) per pass of up to 8 rows, not one per part
    passes = (M + 7) // 8
    assert group_launches <= 2 * passes
    whole = s.matmul_nbits("qkv", a)
    torch.cuda.synchronize()
    assert torch.equal(whole, torch.cat(outs, dim=1))


def test_group_strict_prefill_and_host(grp):
    import torch
    from onnx_runtime_dart_b200 import _lib
    s, W = grp
    rng = np.random.default_rng(2)
    A = rng.standard_normal((3, K)).astype(np.float32)
    strict = _lib.flags_mode(_lib.MODE_STRICT)
    outs = s.matmul_nbits_group("qkv", A, flags=strict)  # host buffers, whole-op path
    for (name, n), y in zip(PARTS.items(), outs):
        assert np.array_equal(y, s.matmul_nbits(name, A, flags=strict))
    outs = s.matmul_nbits_group("qkv", A)  # host buffers, GEMV path
    for name, y in zip(PARTS, outs):
        assert np.array_equal(y, s.matmul_nbits(name, A))
    ap = torch.randn(512, K, device="cuda")
    f16 = _lib.flags_mode(_lib.MODE_MMA_F16)
    outs = s.matmul_nbits_group("qkv", ap, flags=f16)
    torch.cuda.synchronize()
    for name, y in zip(PARTS, outs):
        assert torch.equal(y, s.matmul_nbits(name, ap, flags=f16))


def test_group_graph_replay_and_drop_parts():
    import torch
    from onnx_runtime_dart_b200 import CudaSession
    from onnx_runtime_dart_b200.workloads import make_nbits_weight
    rng = np.random.default_rng(8)
    with CudaSession(0) as s:
        st = torch.cuda.Stream()
        s.set_stream(st.cuda_stream)
        ref = {}
        a = torch.randn(4, K, device="cuda")
        for name in ("gate", "up"):
            B, sc, z = make_nbits_weight(rng, K, 8192, 128, zero_points=False,
                                         scale_dtype=np.float16)
            s.upload_nbits(name, B, sc, z, k=K, n=8192, block_size=128)
        with torch.cuda.stream(st):
            for name in ("gate", "up"):
                ref[name] = s.matmul_nbits(name, a)
            s.fuse_nbits("gate_up", ["gate", "up"], drop_parts=True)
            with pytest.raises(KeyError):
                s.matmul_nbits("gate", a)
            outs = s.matmul_nbits_group("gate_up", a)
            st.synchronize()
            assert torch.equal(outs[0], ref["gate"]) and torch.equal(outs[1], ref["up"])
            s.graph_begin()
            s.matmul_nbits_group("gate_up", a, outs=outs)
            gid = s.graph_end()
            for o in outs:
                o.zero_()
            s.graph_launch(gid)
            st.synchronize()
            s.graph_drop(gid)
            assert torch.equal(outs[0], ref["gate"]) and torch.equal(outs[1], ref["up"])
