"""Per-op-type device profile (ort_cuda_profile_*), the counterpart of the
reference's ExecutionProfile (lib/src/onnx_graph.dart:22-47): call counts
and cumulative time per op type, sorted by time; and the FFMA probe that
gives the exact mode's CUDA-core roofline."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_profile_counts_calls_per_op_type():
    import torch
    from onnx_runtime_dart_b200 import CudaSession
    from onnx_runtime_dart_b200.workloads import make_nbits_weight
    rng = np.random.default_rng(1)
    K, N = 4096, 8192
    B, sc, z = make_nbits_weight(rng, K, N, 128, zero_points=True, scale_dtype=np.float16)
    with CudaSession(0) as s:
        s.upload_nbits("w", B, sc, z, k=K, n=N, block_size=128)
        s.upload_dense("d", rng.standard_normal((256, 512)).astype(np.float32), trans_b=True)
        a = torch.randn(1, K, device="cuda")
        x = torch.randn(64, 512, device="cuda")
        s.matmul_nbits("w", a)  # first call: plan timing, before profiling
        torch.cuda.synchronize()
        s.profile(True)
        for _ in range(5):
            s.matmul_nbits("w", a)
        for _ in range(3):
            s.gemm("d", x, None)
        y = s.matmul_nbits("w", a)
        s.argmax(y)
        ent = s.profile_entries()
        ops = {op: (n, us) for op, n, us in ent}
        assert ops["MatMulNBits"][0] == 6
        assert ops["Gemm"][0] == 3
        assert ops["ArgMax"][0] == 1
        assert all(us > 0 for _, _, us in ent)
        # sorted by cumulative time, longest first
        assert [us for _, _, us in ent] == sorted((us for _, _, us in ent), reverse=True)
        rep = s.profile_report()
        assert rep.splitlines()[0].split() == ["op", "calls", "ms", "share"]
        assert "MatMulNBits" in rep and rep.splitlines()[-1].startswith("total")
        # disabled: no further records; reset clears
        s.profile(False)
        s.matmul_nbits("w", a)
        assert {op: n for op, n, _ in s.profile_entries()}["MatMulNBits"] == 6
        s.profile_reset()
        assert s.profile_entries() == []


def test_ffma_probe_is_plausible():
    from onnx_runtime_dart_b200 import CudaSession
    with CudaSession(0) as s:
        t = s.probe_ffma_tflops()
    # 148 SMs x 128 FP32 lanes x 2 flops x 1.965 GHz = 74.4 TFLOP/s nominal
    assert 20.0 < t < 80.0, t
