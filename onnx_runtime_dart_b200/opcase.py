"""Runs one MatMulNBits call repeatedly on device buffers and prints its
CUDA-event time per launch: the case to time a single projection, or to put
under a profiler with few launches before the one captured.

    python -m onnx_runtime_dart_b200.opcase --k 4096 --n 128256 --m 1
    python -m onnx_runtime_dart_b200.opcase --k 4096 --n 28672 --m 2048 --mode mma_f16

Weights are seeded random int4 (fp16 scales, packed zero points), as in the
benchmark; the first `--warmup` launches are untimed, then `--reps` launches
run back to back between two events (recorded as one CUDA graph with
`--graph`, so that the host's per-call cost stays out of the time).  The
session's error word is read after the timed launches, so an expired
in-kernel wait fails the run.
"""
from __future__ import annotations

import argparse
import json

import numpy as np


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--k", type=int, required=True)
    ap.add_argument("--n", type=int, required=True)
    ap.add_argument("--m", type=int, default=1)
    ap.add_argument("--block-size", type=int, default=128)
    ap.add_argument("--mode", default="exact", choices=["exact", "strict", "mma_f16", "mma_bf16"])
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--reps", type=int, default=5)
    ap.add_argument("--seed", type=int, default=5)
    ap.add_argument("--graph", action="store_true",
                    help="record the timed launches as one CUDA graph and replay it once "
                         "(device time without the host's per-call cost)")
    ap.add_argument("--plan", type=int, default=None,
                    help="decode-GEMV plan to use (ort_cuda_gemv_plan_set) instead of timing "
                         "the candidates on the first call; M <= 8 in the exact mode")
    args = ap.parse_args(argv)

    import torch
    from . import _lib
    from .session import CudaSession
    from .workloads import make_nbits_weight

    s = CudaSession(0, mode=args.mode)
    try:
        st = torch.cuda.Stream()
        s.set_stream(st.cuda_stream)
        rng = np.random.default_rng(args.seed)
        B, sc, z = make_nbits_weight(rng, args.k, args.n, args.block_size, zero_points=True,
                                     scale_dtype=np.float16)
        s.upload_nbits("w", B, sc, z, k=args.k, n=args.n, block_size=args.block_size)
        if args.plan is not None:
            s.set_gemv_plan("w", args.m, args.plan)
        flags = _lib.flags_mode(_lib.MODES[args.mode])
        with torch.cuda.stream(st):
            gen = torch.Generator(device="cuda").manual_seed(args.seed)
            a = torch.randn(args.m, args.k, device="cuda", generator=gen)
            y = torch.empty(args.m, args.n, device="cuda")
            for _ in range(args.warmup):
                s.matmul_nbits("w", a, out=y, flags=flags)
            st.synchronize()
            gid = None
            if args.graph:
                s.graph_begin()
                for _ in range(args.reps):
                    s.matmul_nbits("w", a, out=y, flags=flags)
                gid = s.graph_end()
                s.graph_launch(gid)  # warm replay
                st.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            if gid is not None:
                s.graph_launch(gid)
            else:
                for _ in range(args.reps):
                    s.matmul_nbits("w", a, out=y, flags=flags)
            e1.record(st)
            st.synchronize()
            if gid is not None:
                s.graph_drop(gid)
        s.sync()
        us = e0.elapsed_time(e1) * 1000 / args.reps
        plan = s.gemv_plan("w", args.m) if args.mode == "exact" and args.m <= 8 else None
        print(json.dumps({"op": "MatMulNBits", "k": args.k, "n": args.n, "m": args.m,
                          "block_size": args.block_size, "mode": args.mode, "gemv_plan": plan,
                          "us_per_launch": us, "reps": args.reps,
                          "tflops": 2 * args.m * args.k * args.n / (us * 1e-6) / 1e12}))
    finally:
        s.close()


if __name__ == "__main__":
    main()
