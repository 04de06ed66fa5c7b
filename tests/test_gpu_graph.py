"""CUDA graphs of device-pointer call sequences (ort_cuda_graph_*).

A decode step is a fixed sequence of matmuls on fixed device buffers; the
session records it once and replays it with one launch.  Replays must give
the same bits as running the calls one by one, on new input values written
into the same buffers, for every kernel family the step can contain: the
split-K and the tile-major decode GEMV and the 16-bit prefill GEMM.
"""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture
def tsess():
    import torch
    from onnx_runtime_dart_b200 import CudaSession
    s = CudaSession(0)
    st = torch.cuda.Stream()
    s.set_stream(st.cuda_stream)
    yield s, st
    s.close()


def test_graph_replay_is_bitwise_eager(tsess):
    import torch
    from onnx_runtime_dart_b200 import _lib
    s, st = tsess
    rng = np.random.default_rng(41)
    # x[1, 4096] -> h[1, 6144] (split-K) -> y[1, 50000] (tile-major),
    # and a [256, 1024] prefill in the fp16 MMA mode
    for name, K, N, bs in [("a", 4096, 6144, 128), ("b", 6144, 50000, 32), ("c", 1024, 3000, 64)]:
        B, sc, z = O.make_nbits_weight(rng, K, N, bs, zero_points=True)
        s.upload_nbits(name, B, sc, z, k=K, n=N, block_size=bs)
    f16 = _lib.flags_mode(_lib.MODES["mma_f16"])
    with torch.cuda.stream(st):
        x = torch.empty(1, 4096, device="cuda")
        h = torch.empty(1, 6144, device="cuda")
        y = torch.empty(1, 50000, device="cuda")
        p = torch.empty(256, 1024, device="cuda")
        q = torch.empty(256, 3000, device="cuda")

    def run():
        s.matmul_nbits("a", x, out=h)
        s.matmul_nbits("b", h, out=y)
        s.matmul_nbits("c", p, out=q, flags=f16)

    def fill(seed):
        g = np.random.default_rng(seed)
        x.copy_(torch.from_numpy(g.standard_normal((1, 4096)).astype(np.float32)))
        p.copy_(torch.from_numpy(g.standard_normal((256, 1024)).astype(np.float32)))

    with torch.cuda.stream(st):
        fill(1)
        run()  # every op once before capture
        st.synchronize()
        s.graph_begin()
        run()
        gid = s.graph_end()
        launches = s.launch_count()
        for seed in (2, 3):
            fill(seed)
            run()
            st.synchronize()
            eager = [t.clone() for t in (h, y, q)]
            fill(seed)
            s.graph_launch(gid)
            st.synchronize()
            for a, b in zip(eager, (h, y, q)):
                assert torch.equal(a, b)
        # the replay counted the kernels it holds, as the eager calls do
        per_call = (s.launch_count() - launches) // 4
        assert per_call > 0
        s.graph_drop(gid)


def test_graph_capture_refuses_growth_and_host_io(tsess):
    import torch
    from onnx_runtime_dart_b200 import _lib
    s, st = tsess
    rng = np.random.default_rng(42)
    B, sc, z = O.make_nbits_weight(rng, 1024, 2048, 32, zero_points=False)
    s.upload_nbits("w", B, sc, z, k=1024, n=2048, block_size=32)
    with torch.cuda.stream(st):
        x = torch.randn(1, 1024, device="cuda")
        y = torch.empty(1, 2048, device="cuda")
        s.matmul_nbits("w", x, out=y)
        f16 = _lib.flags_mode(_lib.MODES["mma_f16"])
        small = torch.randn(256, 1024, device="cuda")
        s.matmul_nbits("w", small, out=torch.empty(256, 2048, device="cuda"), flags=f16)
        big = torch.randn(4096, 1024, device="cuda")
        out = torch.empty(4096, 2048, device="cuda")
        st.synchronize()
        s.graph_begin()
        with pytest.raises(ValueError):
            s.matmul_nbits("w", np.ones((1, 1024), np.float32))  # host buffers
        with pytest.raises(ValueError):
            s.matmul_nbits("w", big, out=out, flags=f16)  # would grow the scratch
        s.matmul_nbits("w", x, out=y)
        gid = s.graph_end()
        s.graph_launch(gid)
        st.synchronize()
        ref = O.matmul_nbits(x.cpu().numpy(), B, sc, z, 1024, 2048, 4, 32)
        assert np.abs(y.cpu().numpy() - ref).max() / np.abs(ref).max() <= 1e-5
        with pytest.raises(KeyError):
            s.graph_launch(gid + 100)  # unknown id
