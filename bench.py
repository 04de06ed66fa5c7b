#!/usr/bin/env python
"""MatMulNBits decode benchmark (B200) — one JSON line on rank 0.

Workload (`config.workload`): one decode step of Llama-3-8B-shaped int4
projections at M=1 — qkv 4096->6144, o 4096->4096, gate_up 4096->28672,
down 14336->4096, lm_head 4096->128256 — bits 4, block 128, fp16 scales,
packed uint4 zero points, random-init weights (seed 5), A ~ N(0,1).
Weights are uploaded once; activations stay on the device.  With N GPUs
the output columns of every weight are sharded over the ranks and Y is
all-gathered inside each op, over peer memory (NCCL where peers cannot be
mapped) (strong scaling: total work fixed).  Each op's work plan is timed
and chosen on its first (warm-up) call.

Timing: the K steps are recorded as one CUDA graph and replayed once
between two events; `roofline` times the lm_head op with an event pair
around it in a second replay of the same K steps (events between kernels
end their programmatic overlap, so they stay out of the timed replay).

`value` = whole-job algorithmic bytes per step / device time per step
(max over ranks), GB/s.  Algorithmic bytes per op = packed B + scales +
zero points + 4*M*K (A) + 4*M*N_local (Y), summed over ranks.
`e2e` = the same metric through the C ABI with host buffers (pinned), the
host<->device copies inside the timed region.
`prefill` = the metric's second half: the same five projections at M=2048
in the fp16 tensor-core mode (the mode held to 2e-3 max-relative error),
2*M*K*N flops per op over device time, TFLOP/s, whole job.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "MatMulNBits eff. HBM GB/s (M=1) and TFLOP/s (M=2048) at 1/2/4/8 B200"
BS = 128
SEED = 5
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
PREFILL_M = 2048


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--mode", default="exact", choices=["exact", "mma_f16", "mma_bf16"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="CPU-baseline time budget (rank 0, N=1)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--eager", action="store_true",
                    help="time op-by-op calls instead of a CUDA graph of the timed steps")
    ap.add_argument("--save-plans", default=None,
                    help="write the decode-GEMV plans chosen in warm-up to this JSON file "
                         "(per rank: .rankR appended when N > 1)")
    ap.add_argument("--load-plans", default=None,
                    help="use the plans of a --save-plans file instead of timing them")
    return ap.parse_args()


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def tensor_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["bf16_tflops"]), "measured (burst bf16 GEMM)"
    return FALLBACK_BF16_TFLOPS, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.2)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = [r.split(",") for r in open(self.path).read().strip().splitlines() if r.strip()]
        os.unlink(self.path)
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = max(mx, float(r[2]))
                for nm, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(nm)
            except (ValueError, IndexError):
                continue
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def make_weights(projs):
    from onnx_runtime_dart_b200.workloads import make_nbits_weight
    rng = np.random.default_rng(SEED)
    return {p.name: make_nbits_weight(rng, p.K, p.N, BS, zero_points=True,
                                      scale_dtype=np.float16) for p in projs}


def cpu_sample(projs, weights, budget_s, threads):
    """The reference arithmetic (CPU oracle, port of the Dart path) on a
    bounded sample of the same workload: every projection at M=1 with its
    first min(N, 4096) output columns, repeated for about `budget_s`."""
    from oracle import oracle as O
    from onnx_runtime_dart_b200.workloads import nbits_bytes
    rng = np.random.default_rng(SEED + 1)
    samples = []
    for p in projs:
        B, s, z = weights[p.name]
        nb = p.K // BS
        n = min(p.N, 4096)
        zv = np.stack([z & 0xF, z >> 4], 1).ravel()[:p.N * nb]
        zs = (zv[:n * nb:2] | (zv[1:n * nb:2] << 4)).astype(np.uint8)
        samples.append((p.K, n, np.ascontiguousarray(B[:n]), s[:n * nb].astype(np.float32), zs,
                        rng.standard_normal((1, p.K)).astype(np.float32)))
    bytes_per = sum(nbits_bytes(K, n, BS, 1, 2, True) for K, n, *_ in samples)
    t0 = time.perf_counter()
    reps = 0
    while True:
        for K, n, B, s, z, A in samples:
            O.matmul_nbits(A, B, s, z, K, n, 4, BS, threads=threads)
        reps += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = time.perf_counter() - t0
    return reps * bytes_per / dt / 1e9, reps, dt, bytes_per


def run_reference(args):
    """--impl reference: the reference's CPU arithmetic (oracle port; the
    Dart VM is not installed) on the host cores, rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from onnx_runtime_dart_b200.workloads import LLAMA3_8B
    threads = os.cpu_count() or 1
    weights = make_weights(LLAMA3_8B)
    budget = 2.0
    for _ in range(args.warmup):
        cpu_sample(LLAMA3_8B, weights, 0.0, threads)
    vals, t_all = [], 0.0
    for _ in range(args.steps):
        v, reps, dt, b = cpu_sample(LLAMA3_8B, weights, 0.0, threads)
        vals.append(v)
        t_all += dt
    value = statistics.median(vals)
    sample = ("per step: qkv,o,gate_up,down,lm_head at M=1 on their first min(N,4096) "
              "columns (C restatement of the reference's dequant + SIMD GEMM; Dart VM absent)")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1000 * t_all / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "cfg5 decode M=1 Llama-3-8B int4 projections (column sample)",
                       "parallelism": "host threads (column split)"},
            "cpu_baseline": {"value": value, "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
        return
    assert args.warmup >= 3, "at least 3 warm-up steps"
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    assert world == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE {world}"

    import torch
    import torch.distributed as dist
    from onnx_runtime_dart_b200 import CudaSession
    from onnx_runtime_dart_b200.workloads import LLAMA3_8B, nbits_bytes, shard_range

    torch.cuda.set_device(local)
    nccl_id = None
    if world > 1:
        import datetime
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=120))
        obj = [CudaSession.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        nccl_id = obj[0]
    sess = CudaSession(local, mode=args.mode, rank=rank, world=world, nccl_id=nccl_id,
                       timeout_ms=120000)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    sess.set_stream(stream.cuda_stream)

    projs = LLAMA3_8B
    weights = make_weights(projs)
    for p in projs:
        B, s, z = weights[p.name]
        sess.upload_nbits(p.name, B, s, z, k=p.K, n=p.N, block_size=BS)
    M = 1
    suffix = f".rank{rank}" if world > 1 else ""
    if args.load_plans:
        for name, plan in json.load(open(args.load_plans + suffix)).items():
            sess.set_gemv_plan(name, M, int(plan))
    dev = torch.device("cuda", local)
    gen = torch.Generator(device=dev).manual_seed(SEED)
    A = {K: torch.randn(M, K, device=dev, generator=gen) for K in sorted({p.K for p in projs})}
    Y = {p.name: torch.empty(M, p.N, device=dev) for p in projs}

    # algorithmic bytes this rank moves per step (its column shard)
    rank_bytes = 0
    for p in projs:
        a, b = shard_range(p.N, rank, world)
        rank_bytes += nbits_bytes(p.K, b - a, BS, M, 2, True)
    big = max(projs, key=lambda p: p.K * p.N)
    ba, bb = shard_range(big.N, rank, world)
    big_bytes = nbits_bytes(big.K, bb - ba, BS, M, 2, True)

    def record(event):
        # inside a capture, an external event node: recorded on every replay
        # and readable with elapsed_time, like a plain record
        if capturing[0]:
            from cuda.bindings import runtime as rt
            err, = rt.cudaEventRecordWithFlags(event.cuda_event, stream.cuda_stream,
                                               rt.cudaEventRecordExternal)
            assert int(err) == 0, err
        else:
            event.record(stream)

    capturing = [False]

    def step(ev=None):
        for p in projs:
            if ev is not None and p.name == big.name:
                record(ev[0])
            sess.matmul_nbits(p.name, A[p.K], out=Y[p.name])
            if ev is not None and p.name == big.name:
                record(ev[1])

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        step()
    barrier()
    plans = {p.name: sess.gemv_plan(p.name, M) for p in projs}
    if args.save_plans:
        with open(args.save_plans + suffix, "w") as f:
            json.dump(plans, f)
    clocks = ClockSampler(local)
    clocks.start()
    barrier()
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # Two replays of the same K steps.  The timed one has no events inside
    # (an event between two kernels ends their programmatic overlap); the
    # second records an event pair around each step's lm_head GEMV for the
    # roofline.  Eager mode runs the same two passes op by op.
    gid = gid_ev = None
    if not args.eager:
        for a, b in kev:  # torch creates its events on first use
            a.record(stream)
            b.record(stream)
        barrier()
        sess.graph_begin()
        for i in range(args.steps):
            step()
        gid = sess.graph_end()
        sess.graph_begin()
        capturing[0] = True
        for i in range(args.steps):
            step(kev[i])
        capturing[0] = False
        gid_ev = sess.graph_end()
        sess.graph_launch(gid)  # one untimed replay
        barrier()
    launches0 = sess.launch_count()
    e0.record(stream)
    if gid is not None:
        sess.graph_launch(gid)
    else:
        for i in range(args.steps):
            step()
    e1.record(stream)
    barrier()
    launches = sess.launch_count() - launches0
    if gid_ev is not None:
        sess.graph_launch(gid_ev)
    else:
        for i in range(args.steps):
            step(kev[i])
    barrier()
    for g in (gid, gid_ev):
        if g is not None:
            sess.graph_drop(g)
    sess.sync()  # raises if any kernel of the timed steps reported an error
    clk = clocks.stop()
    ms_step = e0.elapsed_time(e1) / args.steps
    big_ms = sum(a.elapsed_time(b) for a, b in kev) / args.steps

    # ---- prefill: M=2048 in the fp16 tensor-core mode ---------------------
    from onnx_runtime_dart_b200 import _lib
    pf_flags = _lib.flags_mode(_lib.MODES["mma_f16"])
    Ap = {K: torch.randn(PREFILL_M, K, device=dev, generator=gen) for K in A}
    Yp = {p.name: torch.empty(PREFILL_M, p.N, device=dev) for p in projs}

    def step_prefill(ev=None):
        for p in projs:
            if ev is not None and p.name == big.name:
                ev[0].record(stream)
            sess.matmul_nbits(p.name, Ap[p.K], out=Yp[p.name], flags=pf_flags)
            if ev is not None and p.name == big.name:
                ev[1].record(stream)

    pf_steps = max(1, min(args.steps, 10))
    for _ in range(args.warmup):
        step_prefill()
    barrier()
    pev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(pf_steps)]
    e0.record(stream)
    for i in range(pf_steps):
        step_prefill(pev[i])
    e1.record(stream)
    barrier()
    sess.sync()
    pf_ms = e0.elapsed_time(e1) / pf_steps
    pf_big_ms = sum(a.elapsed_time(b) for a, b in pev) / pf_steps
    rank_flops = 0
    for p in projs:
        a, b = shard_range(p.N, rank, world)
        rank_flops += 2 * PREFILL_M * p.K * (b - a)
    ba, bb = shard_range(big.N, rank, world)
    big_flops = 2 * PREFILL_M * big.K * (bb - ba)
    del Ap, Yp

    # ---- cfg4: one decode step of the Llama-3.2-1B matmul stream at M=4 ----
    # 16 distinct layers x (q, k, v, o, gate, up, down) + lm_head, about
    # 0.6 GB of int4 weights per step (larger than L2), in a CUDA graph
    from onnx_runtime_dart_b200.workloads import LLAMA32_1B, LLAMA32_1B_LM_HEAD, make_nbits_weight
    M4 = 4
    c4 = [(f"c4.l{layer}.{p.name}", p) for layer in range(16) for p in LLAMA32_1B]
    c4.append(("c4.lm_head", LLAMA32_1B_LM_HEAD))
    rng4 = np.random.default_rng(SEED + 4)
    for name, p in c4:
        B4, s4, _ = make_nbits_weight(rng4, p.K, p.N, BS, zero_points=False,
                                      scale_dtype=np.float16)
        sess.upload_nbits(name, B4, s4, None, k=p.K, n=p.N, block_size=BS)
    A4 = {K: torch.randn(M4, K, device=dev, generator=gen) for K in sorted({p.K for _, p in c4})}
    Y4 = {name: torch.empty(M4, p.N, device=dev) for name, p in c4}

    def step4():
        for name, p in c4:
            sess.matmul_nbits(name, A4[p.K], out=Y4[name])

    for _ in range(args.warmup):
        step4()
    barrier()
    g4 = None
    if not args.eager:
        sess.graph_begin()
        step4()
        g4 = sess.graph_end()
        sess.graph_launch(g4)  # one untimed replay
        barrier()
    d4_steps = max(1, min(args.steps, 20))
    e0.record(stream)
    for _ in range(d4_steps):
        if g4 is not None:
            sess.graph_launch(g4)
        else:
            step4()
    e1.record(stream)
    barrier()
    if g4 is not None:
        sess.graph_drop(g4)
    sess.sync()
    d4_ms = e0.elapsed_time(e1) / d4_steps
    rank_bytes4 = 0
    for name, p in c4:
        a, b = shard_range(p.N, rank, world)
        rank_bytes4 += nbits_bytes(p.K, b - a, BS, M4, 2, False)
    for name, _ in c4:
        sess.drop_weight(name)
    del A4, Y4

    # ---- end to end through the C ABI with host buffers -----------------
    hostA = {K: torch.randn(M, K, generator=torch.Generator().manual_seed(K)).pin_memory().numpy()
             for K in A}
    hostY = {p.name: torch.empty(M, p.N).pin_memory().numpy() for p in projs}

    def step_e2e():
        for p in projs:
            sess.matmul_nbits(p.name, hostA[p.K], out=hostY[p.name])

    for _ in range(args.warmup):
        step_e2e()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step_e2e()
    barrier()
    e2e_ms = 1000 * (time.perf_counter() - t0) / args.steps
    h2d = sum(4 * M * p.K for p in projs)
    d2h = sum(4 * M * p.N for p in projs)

    stats = torch.tensor([ms_step, e2e_ms, big_ms, pf_ms, pf_big_ms, d4_ms], dtype=torch.float64)
    tot = torch.tensor([rank_bytes, launches, rank_flops, rank_bytes4], dtype=torch.float64)
    if world > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
        dist.all_reduce(tot, op=dist.ReduceOp.SUM)
    ms_step, e2e_ms, big_ms, pf_ms, pf_big_ms, d4_ms = stats.tolist()
    job_bytes, launches, job_flops, job_bytes4 = tot.tolist()

    if rank == 0:
        peak, peak_kind = peaks()
        tpk, tpk_kind = tensor_peak()
        achieved = big_bytes / (big_ms * 1e-3) / 1e9
        traffic = None
        tp = os.path.join(ROOT, "profiles", "gemv_lm_head_traffic.json")
        if os.path.exists(tp):
            traffic = json.load(open(tp)).get("dram_bytes_per_launch")
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            threads = os.cpu_count() or 1
            v, reps, dt, b = cpu_sample(projs, weights, args.cpu_seconds, threads)
            cpu = {"value": v, "unit": "GB/s", "cores": threads, "kind": "port",
                   "sample": f"{reps} reps x (qkv,o,gate_up,down,lm_head at M=1 on their first "
                             f"min(N,4096) columns, {b} B each) in {dt:.1f} s; C restatement of "
                             "the reference's dequant + SIMD GEMM (Dart VM absent)"}
        line = {
            "metric": METRIC, "value": job_bytes / (ms_step * 1e-3) / 1e9, "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (random-init Llama-3-8B-shaped int4 weights, seed 5)",
            "config": {"workload": "cfg5 decode step at M=1: MatMulNBits qkv 4096x6144, o "
                                   "4096x4096, gate_up 4096x28672, down 14336x4096, lm_head "
                                   "4096x128256; bits 4, block 128, fp16 scales, packed zp",
                       "mode": args.mode,
                       "gemv_plans": plans,
                       "launch": ("op-by-op calls" if args.eager else
                                  "CUDA graph of the timed steps, one replay"),
                       "parallelism": f"N-sharded x{world}" + (
                           " + all-gather of Y over peer memory (NCCL where peers cannot "
                           "be mapped)" if world > 1 else ""),
                       "l2": "inputs larger than L2 (about 387 MB of weights per step)"},
            "roofline": {"bound": "hbm",
                         "kernel": f"int4 GEMV op ({big.name}: the GEMV launch, plus the "
                                   "chunk-sum launch when its tuned plan is split-K)",
                         "timing": "event pair around the op in a second replay of the steps",
                         "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind,
                         "traffic": traffic, "bytes_per_launch": big_bytes},
            "cpu_baseline": cpu,
            "e2e": {"value": job_bytes / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": e2e_ms},
            "gpu_launches": int(launches),
            "clocks": clk,
            "prefill": {
                "value": job_flops / (pf_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                "M": PREFILL_M, "mode": "mma_f16", "ms_per_step": pf_ms, "steps": pf_steps,
                "roofline": {"bound": "tensor", "kernel": f"int4 dequant + tcgen05 GEMM ({big.name})",
                             "achieved": big_flops / (pf_big_ms * 1e-3) / 1e12,
                             "peak": tpk, "unit": "TFLOP/s",
                             "frac": big_flops / (pf_big_ms * 1e-3) / 1e12 / tpk,
                             "peak_kind": tpk_kind},
            },
            "decode_m4": {
                "value": job_bytes4 / (d4_ms * 1e-3) / 1e9, "unit": "GB/s", "M": M4,
                "mode": args.mode, "ms_per_step": d4_ms, "steps": d4_steps,
                "frac": job_bytes4 / (d4_ms * 1e-3) / 1e9 / peak, "peak_kind": peak_kind,
                "workload": "cfg4 decode step: Llama-3.2-1B int4 matmul stream, 16 layers x "
                            "(q 2048x2048, k/v 2048x512, o 2048x2048, gate/up 2048x8192, "
                            "down 8192x2048) + lm_head 2048x128256 at M=4; bits 4, block 128, "
                            "fp16 scales, no zero points; CUDA graph of one step, weights "
                            f"{job_bytes4 / 1e6:.0f} MB per step (larger than L2)"},
        }
        print(json.dumps(line), flush=True)
    sess.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
