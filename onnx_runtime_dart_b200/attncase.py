"""Runs one GroupQueryAttention call repeatedly on device buffers and prints
its CUDA-event time per launch, with the algorithmic bytes and flops: the
case to time the attention of a decode or prefill step, or to put under a
profiler with few launches before the one captured.

    python -m onnx_runtime_dart_b200.attncase --batch 4 --seq 1 --past 639
    python -m onnx_runtime_dart_b200.attncase --batch 1 --seq 4096 --past 0 --head 128

Inputs are seeded random Q/K/V with RoPE from random cos/sin caches; the KV
cache is in place (present = past buffer of capacity past + seq), as a
decode loop keeps it.  Each timed launch is preceded by a write of a 256 MiB
buffer (larger than L2) so that the cache is read from HBM, as it is when
the projections of a layer run between two attention calls.  Algorithmic
bytes: past K and V read, Q/K/V of the step read, output and the step's
present rows written; flops 4*H*D per (query, visible key) pair.
"""
from __future__ import annotations

import argparse
import json

import numpy as np


def algorithmic(batch, seq, past, heads, kv_heads, head):
    """(bytes, flops) of one GroupQueryAttention call with an in-place cache."""
    f = 4
    bytes_ = (2 * batch * kv_heads * past * head * f            # past K, V
              + batch * seq * (heads + 2 * kv_heads) * head * f  # Q, K, V of the step
              + batch * seq * heads * head * f                   # output
              + 2 * batch * kv_heads * seq * head * f)           # present rows
    pairs = batch * (seq * past + seq * (seq + 1) // 2)          # causal (query, key)
    return bytes_, 4 * heads * head * pairs


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--batch", type=int, default=4)
    ap.add_argument("--seq", type=int, default=1)
    ap.add_argument("--past", type=int, default=639)
    ap.add_argument("--heads", type=int, default=32)
    ap.add_argument("--kv-heads", type=int, default=8)
    ap.add_argument("--head", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--no-flush", action="store_true", help="no L2 flush between launches")
    ap.add_argument("--seed", type=int, default=5)
    args = ap.parse_args(argv)

    import torch
    from . import _lib
    from .session import CudaSession

    B, S, P, H, Hkv, D = args.batch, args.seq, args.past, args.heads, args.kv_heads, args.head
    cap = P + S
    s = CudaSession(0)
    try:
        st = torch.cuda.Stream()
        s.set_stream(st.cuda_stream)
        with torch.cuda.stream(st):
            g = torch.Generator(device="cuda").manual_seed(args.seed)
            q = torch.randn(B, S, H * D, device="cuda", generator=g)
            k = torch.randn(B, S, Hkv * D, device="cuda", generator=g)
            v = torch.randn(B, S, Hkv * D, device="cuda", generator=g)
            kc = torch.randn(B, Hkv, cap, D, device="cuda", generator=g)
            vc = torch.randn(B, Hkv, cap, D, device="cuda", generator=g)
            ang = torch.rand(cap, D // 2, device="cuda", generator=g) * 6.3
            cos, sin = torch.cos(ang), torch.sin(ang)
            flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")

            out = torch.empty(B, S, H * D, device="cuda")
            L = _lib.load()
            argv_c = (s.handle, q.data_ptr(), k.data_ptr(), v.data_ptr(), kc.data_ptr(),
                      vc.data_ptr(), B, S, P, H, Hkv, D, 0.0, cos.data_ptr(), sin.data_ptr(),
                      D // 2, cap, None, 0, 0, cap, out.data_ptr(), kc.data_ptr(),
                      vc.data_ptr(), _lib.ROTARY)

            def call():  # the C ABI with resolved pointers: no Python work in the timing
                _lib.check(L.ort_cuda_group_query_attention(*argv_c),
                           "ort_cuda_group_query_attention")

            l0 = s.launch_count()
            for _ in range(args.warmup):
                call()
            st.synchronize()
            per_call = (s.launch_count() - l0) // max(1, args.warmup)
            times = []
            for _ in range(args.reps):
                if not args.no_flush:
                    flush.fill_(1)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(st)
                call()
                e1.record(st)
                e1.synchronize()
                times.append(e0.elapsed_time(e1) * 1e3)
        us = float(np.median(times))
        nbytes, flops = algorithmic(B, S, P, H, Hkv, D)
        print(json.dumps({"op": "GroupQueryAttention", "batch": B, "seq": S, "past": P,
                          "heads": H, "kv_heads": Hkv, "head": D, "us_median": round(us, 3),
                          "us_min": round(min(times), 3), "launches_per_call": per_call,
                          "bytes": nbytes, "flops": flops,
                          "GB_per_s": round(nbytes / us / 1e3, 1),
                          "TFLOP_per_s": round(flops / us / 1e6, 2),
                          "l2_flush": not args.no_flush}))
    finally:
        s.close()


if __name__ == "__main__":
    main()
