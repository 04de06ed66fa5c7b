#!/usr/bin/env python
"""MatMulNBits / Gemm benchmark (B200) — one JSON line on rank 0.

Headline workload (`config.workload`): one decode step of Llama-3-8B-shaped
int4 projections at M=1 — qkv 4096->6144, o 4096->4096, gate_up 4096->28672,
down 14336->4096, lm_head 4096->128256 — bits 4, block 128, fp16 scales,
packed uint4 zero points, random-init weights (seed 5), A ~ N(0,1).
Weights are uploaded once; activations stay on the device.  With N GPUs
the output columns of every weight are sharded over the ranks and Y is
exchanged inside each op over peer memory (strong scaling: total work
fixed).  Each op's work plan is timed and chosen on its first (warm-up)
call.

Timing: the K steps are recorded as one CUDA graph and replayed once
between two events; `roofline` times the lm_head op with an event pair
around it in a second replay of the same K steps (events between kernels
end their programmatic overlap, so they stay out of the timed replay).

`value` = algorithmic bytes of the step / device time per step (max over
ranks), GB/s.  Algorithmic bytes per op = packed B + scales + zero points +
4*M*K (A) + 4*M*N (Y), counted once per op whatever N is.
`e2e` = the same metric through the C ABI (ort_cuda_matmul_nbits with
ORT_CUDA_HOST_IO on pinned host buffers), host<->device copies inside the
timed region.
`prefill` = the metric's second half: the same five projections at M=2048
in the fp16 tensor-core mode (the mode held to 2e-3 max-relative error),
2*M*K*N flops per op over device time, TFLOP/s, whole job.
`configs` = every other named configuration (cfg1 .. cfg5), each with its
rate, its roofline fraction and, at N=1, the CPU baseline beside it.
`sharded_parity` (N > 1) = the sharded results of the headline ops (M=1,
exact mode) and of the prefill ops (M=2048, fp16 mode) against a
single-GPU session of the same weights on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
"""
from __future__ import annotations

import argparse
import ctypes
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
L2_FLUSH_BYTES = 256 << 20  # written between timed steps of L2-resident configs


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--mode", default="exact", choices=["exact", "mma_f16", "mma_bf16"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="CPU-baseline time budget of the headline (rank 0, N=1)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-configs", action="store_true",
                    help="time only the headline, prefill and e2e legs")
    ap.add_argument("--eager", action="store_true",
                    help="time op-by-op calls instead of a CUDA graph of the timed steps")
    ap.add_argument("--save-plans", default=None,
                    help="write the decode-GEMV plans chosen in warm-up to this JSON file "
                         "(per rank: .rankR appended when N > 1)")
    ap.add_argument("--load-plans", default=None,
                    help="use the plans of a --save-plans file instead of timing them")
    return ap.parse_args()


def _peaks_file():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    return json.load(open(p)) if os.path.exists(p) else None


def peaks():
    d = _peaks_file()
    if d:
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def tensor_peak():
    d = _peaks_file()
    if d:
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


def make_weights(projs, bs=BS, seed=SEED, zero_points=True, scale_dtype=np.float16):
    from onnx_runtime_dart_b200.workloads import make_nbits_weight
    rng = np.random.default_rng(seed)
    return {p.name: make_nbits_weight(rng, p.K, p.N, bs, zero_points=zero_points,
                                      scale_dtype=scale_dtype) for p in projs}


def _column_sample(p, weights, bs, ncols, rng, M=1):
    """The first ncols output columns of projection p (B rows, scales, flat
    zero points re-packed) and an A of M rows: a bounded CPU sample."""
    B, s, z = weights[p.name]
    nb = (p.K + bs - 1) // bs
    n = min(p.N, ncols)
    zs = None
    if z is not None:
        zv = np.stack([z & 0xF, z >> 4], 1).ravel()[:p.N * nb]
        zs = (zv[:n * nb:2] | (zv[1:n * nb:2] << 4)).astype(np.uint8)
    return (p.K, n, np.ascontiguousarray(B[:n]), s[:n * nb].astype(np.float32), zs,
            rng.standard_normal((M, p.K)).astype(np.float32))


def cpu_rate(run_once, units_per_run, budget_s):
    """Repeats run_once() for about budget_s (at least once): units per second."""
    t0 = time.perf_counter()
    reps = 0
    while True:
        run_once()
        reps += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = time.perf_counter() - t0
    return reps * units_per_run / dt, reps, dt


def cpu_sample(projs, weights, budget_s, threads, bs=BS, ncols=4096, M=1, scale_bytes=2):
    """The reference arithmetic (CPU oracle, port of the Dart path) on a
    bounded sample of the same workload: every projection at M rows with
    its first min(N, ncols) output columns, repeated for about `budget_s`."""
    from oracle import oracle as O
    from onnx_runtime_dart_b200.workloads import nbits_bytes
    rng = np.random.default_rng(SEED + 1)
    samples = [_column_sample(p, weights, bs, ncols, rng, M) for p in projs]
    has_zp = any(z is not None for _, _, _, _, z, _ in samples)
    bytes_per = sum(nbits_bytes(K, n, bs, M, scale_bytes, has_zp) for K, n, *_ in samples)

    def once():
        for K, n, B, s, z, A in samples:
            O.matmul_nbits(A, B, s, z, K, n, 4, bs, threads=threads)

    v, reps, dt = cpu_rate(once, bytes_per, budget_s)
    return v / 1e9, reps, dt, bytes_per


def run_reference(args):
    """--impl reference: the reference's CPU arithmetic (oracle port; the
    Dart VM is not installed) on the host cores, rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from onnx_runtime_dart_b200.workloads import LLAMA3_8B
    threads = os.cpu_count() or 1
    weights = make_weights(LLAMA3_8B)
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


class Bench:
    """Device-side timing helpers shared by the legs (one session, one
    stream; under torchrun every rank runs every leg)."""

    def __init__(self, sess, stream, dev, rank, world, dist):
        import torch
        self.torch = torch
        self.sess, self.stream, self.dev = sess, stream, dev
        self.rank, self.world, self.dist = rank, world, dist
        self.flush_buf = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
        self.flush_read = torch.zeros(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)

    def flush_l2(self):
        """Writes a buffer twice the size of L2, then reads another one, so
        the timed step starts with neither its inputs nor dirty lines (whose
        write-back would be charged to it) in L2."""
        self.flush_buf.zero_()
        self.flush_read.sum()

    def barrier(self):
        self.torch.cuda.synchronize()
        if self.world > 1:
            self.dist.barrier()

    def max_over_ranks(self, vals):
        t = self.torch.tensor(vals, dtype=self.torch.float64)
        if self.world > 1:
            self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return t.tolist()

    def graph(self, fn):
        """Runs fn() once eagerly (plans, buffers), then records it as a graph."""
        fn()
        self.barrier()
        self.sess.graph_begin()
        fn()
        return self.sess.graph_end()

    def time_graph(self, gid, reps, flush):
        """ms per replay of graph gid.  flush: an L2-sized write before every
        replay and an event pair around each replay only; else one event pair
        around reps back-to-back replays."""
        torch = self.torch
        ev = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731
        self.sess.graph_launch(gid)  # warm replay
        self.barrier()
        if not flush:
            e0, e1 = ev(), ev()
            e0.record(self.stream)
            for _ in range(reps):
                self.sess.graph_launch(gid)
            e1.record(self.stream)
            self.barrier()
            self.sess.sync()
            return e0.elapsed_time(e1) / reps
        pairs = [(ev(), ev()) for _ in range(reps)]
        for a, b in pairs:
            self.flush_l2()
            a.record(self.stream)
            self.sess.graph_launch(gid)
            b.record(self.stream)
        self.barrier()
        self.sess.sync()
        return sum(a.elapsed_time(b) for a, b in pairs) / reps

    def time_fn(self, fn, reps, flush, graph=True):
        """ms per call of fn(): recorded as a CUDA graph, or (graph=False, for
        steps of long kernels) called eagerly between one event pair."""
        if not graph:
            torch = self.torch
            fn()
            self.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(self.stream)
            for _ in range(reps):
                fn()
            e1.record(self.stream)
            self.barrier()
            self.sess.sync()
            return e0.elapsed_time(e1) / reps
        gid = self.graph(fn)
        try:
            return self.time_graph(gid, reps, flush)
        finally:
            self.sess.graph_drop(gid)


def leg_nbits(bench, tag, projs, weights, M, mode, bs, scale_bytes, zp, reps, flush,
              workload, hbm, tpk, cpu=None, per_op=False):
    """One named MatMulNBits configuration: upload, time the step (and each
    op when per_op), report its rate and roofline fraction."""
    torch = bench.torch
    from onnx_runtime_dart_b200 import _lib
    from onnx_runtime_dart_b200.workloads import nbits_bytes, nbits_flops
    sess, dev = bench.sess, bench.dev
    names = []
    for p in projs:
        B, s, z = weights[p.name]
        nm = f"{tag}.{p.name}"
        sess.upload_nbits(nm, B, s, z, k=p.K, n=p.N, block_size=bs)
        names.append((nm, p))
    gen = torch.Generator(device=dev).manual_seed(SEED + M)
    A = {K: torch.randn(M, K, device=dev, generator=gen) for K in sorted({p.K for p in projs})}
    Y = {nm: torch.empty(M, p.N, device=dev) for nm, p in names}
    flags = _lib.flags_mode(_lib.MODES[mode])
    # the C ABI called directly (as a Dart binding would): the Python
    # wrapper's own overhead would otherwise bound the eager prefill legs
    L = _lib.load()
    h = ctypes.c_void_p(sess.handle)
    calls = [(nm.encode(), A[p.K].data_ptr(), Y[nm].data_ptr()) for nm, p in names]

    def step():
        for nb_, a_, y_ in calls:
            rc = L.ort_cuda_matmul_nbits(h, nb_, a_, M, y_, flags)
            if rc:
                _lib.check(rc, "ort_cuda_matmul_nbits")

    bytes_step = sum(nbits_bytes(p.K, p.N, bs, M, scale_bytes, zp) for p in projs)
    flops_step = sum(nbits_flops(p.K, p.N, M) for p in projs)
    # decode steps are recorded as a CUDA graph; prefill-sized steps (long
    # kernels, launch cost negligible) run eagerly
    graph = M <= 16
    ms = bench.time_fn(step, reps, flush, graph=graph)
    ops = {}
    if per_op:
        for nm, p in names:
            ops[p.name] = bench.time_fn(
                lambda nm=nm, p=p: sess.matmul_nbits(nm, A[p.K], out=Y[nm], flags=flags),
                reps, flush, graph=graph)
    vals = bench.max_over_ranks([ms] + [ops[k] for k in sorted(ops)])
    ms, opv = vals[0], dict(zip(sorted(ops), vals[1:]))
    for nm, _ in names:
        sess.drop_weight(nm)
    out = {"workload": workload, "M": M, "mode": mode, "ms_per_step": ms,
           "l2": "flushed (256 MB write, then a 256 MB read) before every timed step" if flush
                 else "weights larger than L2"}
    if mode == "exact" and M <= 16:
        gbs = bytes_step / (ms * 1e-3) / 1e9
        out.update({"value": gbs, "unit": "GB/s", "bound": "hbm", "frac": gbs / hbm,
                    "bytes_per_step": bytes_step})
        if opv:
            out["per_op"] = {k: {"us": 1000 * v,
                                 "GB/s": nbits_bytes(p.K, p.N, bs, M, scale_bytes, zp)
                                 / (v * 1e-3) / 1e9}
                             for k, v in opv.items() for p in projs if p.name == k}
    else:
        tf = flops_step / (ms * 1e-3) / 1e12
        out.update({"value": tf, "unit": "TFLOP/s", "bound": "tensor", "frac": tf / tpk,
                    "flops_per_step": flops_step})
    if cpu is not None:
        out["cpu_baseline"] = cpu
    return out


def leg_cfg4_grouped(bench, c4, w4, M, reps, hbm, tpk=None, mode="exact"):
    """cfg4's step with each layer's sibling projections fused
    (ort_cuda_fuse_nbits: q/k/v and gate/up) and run as one operation each
    (ort_cuda_matmul_nbits_group): 4 operations per layer instead of 7, the
    same weights, bytes and results.  Decode (M=4, exact) or prefill
    (M=2048, fp16)."""
    torch = bench.torch
    from onnx_runtime_dart_b200 import _lib
    from onnx_runtime_dart_b200.workloads import nbits_bytes, nbits_flops
    flags = _lib.flags_mode(_lib.MODES[mode])
    sess, dev = bench.sess, bench.dev
    for p in c4:
        B, s, z = w4[p.name]
        sess.upload_nbits("g." + p.name, B, s, z, k=p.K, n=p.N, block_size=BS)
    steps = []
    for layer in range(16):
        pre = f"g.l{layer}."
        sess.fuse_nbits(pre + "qkv", [pre + "q", pre + "k", pre + "v"], drop_parts=True)
        sess.fuse_nbits(pre + "gate_up", [pre + "gate", pre + "up"], drop_parts=True)
        steps += [("group", pre + "qkv", 2048), ("one", pre + "o", 2048),
                  ("group", pre + "gate_up", 2048), ("one", pre + "down", 8192)]
    steps.append(("one", "g.lm_head", 2048))
    gen = torch.Generator(device=dev).manual_seed(SEED + 40)
    A = {K: torch.randn(M, K, device=dev, generator=gen) for K in (2048, 8192)}
    outs = {}
    for kind, nm, K in steps:
        if kind == "group":
            outs[nm] = sess.matmul_nbits_group(nm, A[K], flags=flags)
        else:
            outs[nm] = sess.matmul_nbits(nm, A[K], flags=flags)

    L = _lib.load()
    h = ctypes.c_void_p(sess.handle)
    calls = []
    for kind, nm, K in steps:
        if kind == "group":
            ptrs = (ctypes.c_void_p * len(outs[nm]))(*[o.data_ptr() for o in outs[nm]])
            calls.append((L.ort_cuda_matmul_nbits_group, nm.encode(), A[K].data_ptr(), ptrs))
        else:
            calls.append((L.ort_cuda_matmul_nbits, nm.encode(), A[K].data_ptr(),
                          outs[nm].data_ptr()))

    def step():
        for fn, nb_, a_, y_ in calls:
            rc = fn(h, nb_, a_, M, y_, flags)
            if rc:
                _lib.check(rc, "matmul_nbits")

    ms = bench.max_over_ranks([bench.time_fn(step, reps, False, graph=M <= 16)])[0]
    for kind, nm, K in steps:
        sess.drop_weight(nm)
    del outs, A
    out = {"workload": f"cfg4 step at M={M} with sibling projections fused: per layer "
                       "qkv (q,k,v) and gate_up (gate,up) as one operation each, o, down; "
                       "plus lm_head (65 operations instead of 113; same weights and results)",
           "M": M, "mode": mode, "ms_per_step": ms}
    if M <= 16:
        bytes_step = sum(nbits_bytes(p.K, p.N, BS, M, 2, False) for p in c4)
        gbs = bytes_step / (ms * 1e-3) / 1e9
        out.update({"value": gbs, "unit": "GB/s", "bound": "hbm", "frac": gbs / hbm,
                    "bytes_per_step": bytes_step, "l2": "weights larger than L2"})
    else:
        flops = sum(nbits_flops(p.K, p.N, M) for p in c4)
        tf = flops / (ms * 1e-3) / 1e12
        out.update({"value": tf, "unit": "TFLOP/s", "bound": "tensor", "frac": tf / tpk,
                    "flops_per_step": flops})
    return out


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
    from onnx_runtime_dart_b200 import CudaSession, _lib
    from onnx_runtime_dart_b200.workloads import (LLAMA3_8B, LLAMA32_1B, LLAMA32_1B_LM_HEAD,
                                                  QWEN3_06B, Proj, make_nbits_weight,
                                                  nbits_bytes, shard_range)

    torch.cuda.set_device(local)
    nccl_id = None
    if world > 1:
        import datetime
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=300))
        obj = [CudaSession.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        nccl_id = obj[0]
    sess = CudaSession(local, mode=args.mode, rank=rank, world=world, nccl_id=nccl_id,
                       timeout_ms=120000)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    sess.set_stream(stream.cuda_stream)
    dev = torch.device("cuda", local)
    bench = Bench(sess, stream, dev, rank, world, dist)
    hbm, hbm_kind = peaks()
    tpk, tpk_kind = tensor_peak()
    threads = os.cpu_count() or 1
    do_cpu = world == 1 and not args.no_cpu_baseline and rank == 0

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
    gen = torch.Generator(device=dev).manual_seed(SEED)
    A = {K: torch.randn(M, K, device=dev, generator=gen) for K in sorted({p.K for p in projs})}
    Y = {p.name: torch.empty(M, p.N, device=dev) for p in projs}

    # algorithmic bytes of the step (each op counted once) and of the lm_head
    # op; the roofline divides this rank's share of the lm_head bytes by its
    # time
    job_bytes = sum(nbits_bytes(p.K, p.N, BS, M, 2, True) for p in projs)
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

    barrier = bench.barrier
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
    job_flops = sum(2 * PREFILL_M * p.K * p.N for p in projs)
    ba, bb = shard_range(big.N, rank, world)
    big_flops = 2 * PREFILL_M * big.K * (bb - ba)
    del Ap, Yp

    # ---- every other named configuration -----------------------------------
    configs = {}
    if not args.no_configs:
        reps_small = max(10, min(args.steps, 50))
        # cfg5 at M=16 (exact GEMV, two passes of 8 rows) and M=4096 (fp16 MMA)
        cpu = None
        if do_cpu:
            v, r, dt, b = cpu_sample(projs, weights, 2.0, threads, ncols=1024, M=16)
            cpu = {"value": v, "unit": "GB/s", "cores": threads, "kind": "port",
                   "sample": f"{r} reps x cfg5 projections at M=16 on their first 1024 columns "
                             f"({b} B) in {dt:.1f} s"}
        configs["cfg5_m16"] = leg_nbits(
            bench, "c5m16", projs, weights, 16, "exact", BS, 2, True, reps_small, False,
            "cfg5 Llama-3-8B projections at M=16 (exact mode)", hbm, tpk, cpu)
        cpu = None
        if do_cpu:
            from oracle import oracle as O
            rng = np.random.default_rng(SEED + 2)
            K0, n0_, Bs_, s_, z_, _ = _column_sample(projs[0], weights, BS, 128, rng)
            Acpu = rng.standard_normal((256, K0)).astype(np.float32)
            fl = 2 * 256 * K0 * n0_
            v, r, dt = cpu_rate(lambda: O.matmul_nbits(Acpu, Bs_, s_, z_, K0, n0_, 4, BS,
                                                       threads=threads), fl, 2.0)
            cpu = {"value": v / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                   "sample": f"{r} reps x qkv at M=256 on 128 columns in {dt:.1f} s"}
        configs["cfg5_m4096"] = leg_nbits(
            bench, "c5m4k", projs, weights, 4096, "mma_f16", BS, 2, True, 3, False,
            "cfg5 Llama-3-8B projections at M=4096 (fp16 tensor-core mode)", hbm, tpk, cpu)

        # cfg3: Qwen3-0.6B decode projections at M=1 (bs 32, fp32 scales, zp)
        q3 = QWEN3_06B
        w3 = make_weights(q3, bs=32, seed=SEED + 3, zero_points=True, scale_dtype=np.float32)
        cpu = None
        if do_cpu:
            v, r, dt, b = cpu_sample(q3, w3, 2.0, threads, bs=32, ncols=4096, scale_bytes=4)
            cpu = {"value": v, "unit": "GB/s", "cores": threads, "kind": "port",
                   "sample": f"{r} reps x the nine projections at M=1 on their first 4096 "
                             f"columns ({b} B) in {dt:.1f} s"}
        configs["cfg3"] = leg_nbits(
            bench, "c3", q3, w3, 1, "exact", 32, 4, True, reps_small, True,
            "cfg3 Qwen3-0.6B decode projections at M=1 (q 1024x2048, k/v 1024x1024, "
            "o 2048x1024, gate/up 1024x3072, down 3072x1024, lm_head 1024x151936); bits 4, "
            "block 32, fp32 scales, packed zp", hbm, tpk, cpu, per_op=True)
        del w3

        # cfg1: one MatMulNBits, M=16, K=N=1024, bs 32, fp32 scales, no zp (seed 0)
        p1 = [Proj("op", 1024, 1024)]
        rng1 = np.random.default_rng(0)
        w1 = {"op": make_nbits_weight(rng1, 1024, 1024, 32, zero_points=False,
                                      scale_dtype=np.float32)}
        cpu = None
        if do_cpu:
            v, r, dt, b = cpu_sample(p1, w1, 1.0, threads, bs=32, ncols=1024, M=16,
                                     scale_bytes=4)
            cpu = {"value": v, "unit": "GB/s", "cores": threads, "kind": "port",
                   "sample": f"{r} reps of the whole op ({b} B) in {dt:.1f} s"}
        configs["cfg1"] = leg_nbits(
            bench, "c1", p1, w1, 16, "exact", 32, 4, False, reps_small, True,
            "cfg1 single MatMulNBits, A [1,16,1024], K=N=1024, bits 4, block 32, fp32 "
            "scales, no zero points", hbm, tpk, cpu)

        # cfg4: Llama-3.2-1B int4 stream: 16 layers x (q,k,v,o,gate,up,down) +
        # lm_head; 128-step decode at M=4 (one step timed per replay) and the
        # prefill at M=2048 in the fp16 mode
        c4 = [Proj(f"l{layer}.{p.name}", p.K, p.N) for layer in range(16) for p in LLAMA32_1B]
        c4.append(LLAMA32_1B_LM_HEAD)
        w4 = make_weights(c4, seed=SEED + 4, zero_points=False)
        cpu = None
        if do_cpu:
            v, r, dt, b = cpu_sample(c4[:7] + [c4[-1]], w4, 2.0, threads, ncols=2048, M=4)
            cpu = {"value": v, "unit": "GB/s", "cores": threads, "kind": "port",
                   "sample": f"{r} reps x one layer's projections + lm_head at M=4 on their "
                             f"first 2048 columns ({b} B) in {dt:.1f} s"}
        configs["cfg4_decode_m4"] = leg_nbits(
            bench, "c4", c4, w4, 4, "exact", BS, 2, False, max(1, min(args.steps, 20)), False,
            "cfg4 decode step: Llama-3.2-1B int4 matmul stream, 16 layers x (q 2048x2048, "
            "k/v 2048x512, o 2048x2048, gate/up 2048x8192, down 8192x2048) + lm_head "
            "2048x128256 at M=4; bits 4, block 128, fp16 scales, no zero points", hbm, tpk,
            cpu)
        configs["cfg4_decode_m4_grouped"] = leg_cfg4_grouped(
            bench, c4, w4, 4, max(1, min(args.steps, 20)), hbm)
        configs["cfg4_prefill_m2048"] = leg_nbits(
            bench, "c4p", c4, w4, PREFILL_M, "mma_f16", BS, 2, False, 3, False,
            "cfg4 prefill: the same 113 projections at M=2048 (4 x 512 tokens), fp16 "
            "tensor-core mode", hbm, tpk)
        configs["cfg4_prefill_m2048_grouped"] = leg_cfg4_grouped(
            bench, c4, w4, PREFILL_M, 3, hbm, tpk, mode="mma_f16")
        del w4

        # cfg2: fp32 Gemm with prepacked B (transB=1, alpha=beta=1) at the
        # BERT-384 FFN shapes, up [1024,384]x[1536,384]^T + bias, then down
        # [1024,1536]x[384,1536]^T + bias (seed 1); exact (FFMA) and fp16 modes
        rng2 = np.random.default_rng(1)
        A1 = rng2.standard_normal((1024, 384)).astype(np.float32)
        W1 = (rng2.standard_normal((1536, 384)) * 0.05).astype(np.float32)
        C1 = (rng2.standard_normal(1536) * 0.02).astype(np.float32)
        A2 = rng2.standard_normal((1024, 1536)).astype(np.float32)
        W2 = (rng2.standard_normal((384, 1536)) * 0.05).astype(np.float32)
        C2 = (rng2.standard_normal(384) * 0.02).astype(np.float32)
        sess.upload_dense("c2.up", W1, trans_b=True)
        sess.upload_dense("c2.down", W2, trans_b=True)
        dA1, dC1 = torch.from_numpy(A1).to(dev), torch.from_numpy(C1).to(dev)
        dA2, dC2 = torch.from_numpy(A2).to(dev), torch.from_numpy(C2).to(dev)
        dY1 = torch.empty(1024, 1536, device=dev)
        dY2 = torch.empty(1024, 384, device=dev)
        flops2 = 2 * 2 * 1024 * 384 * 1536
        ffma = max(bench.max_over_ranks([sess.probe_ffma_tflops()]))
        c2 = {"workload": "cfg2 fp32 Gemm BERT-384 FFN: [1024,384]x[1536,384]^T + bias, then "
                          "[1024,1536]x[384,1536]^T + bias (transB prepacked, alpha=beta=1)",
              "flops_per_step": flops2, "ffma_peak_tflops": ffma,
              "ffma_peak_kind": "measured (ort_cuda_probe_ffma, fp32 FFMA chains)",
              "l2": "flushed (256 MB write, then a 256 MB read) before every timed step"}
        for mode in ("exact", "mma_f16"):
            fl = _lib.flags_mode(_lib.MODES[mode])

            def step2(fl=fl):
                sess.gemm("c2.up", dA1, dC1, flags=fl, out=dY1)
                sess.gemm("c2.down", dA2, dC2, flags=fl, out=dY2)

            ms2 = bench.max_over_ranks([bench.time_fn(step2, reps_small, True)])[0]
            tf = flops2 / (ms2 * 1e-3) / 1e12
            peak = ffma if mode == "exact" else tpk
            c2[mode] = {"value": tf, "unit": "TFLOP/s", "ms_per_step": ms2,
                        "bound": "fp32 FFMA" if mode == "exact" else "tensor",
                        "frac": tf / peak}
        if do_cpu:
            from oracle import oracle as O
            v, r, dt = cpu_rate(lambda: (O.gemm(A1, W1, C1, transB=True, threads=threads),
                                         O.gemm(A2, W2, C2, transB=True, threads=threads)),
                                flops2, 2.0)
            c2["cpu_baseline"] = {"value": v / 1e12, "unit": "TFLOP/s", "cores": threads,
                                  "kind": "port",
                                  "sample": f"{r} reps of the whole up+down step in {dt:.1f} s"}
        sess.drop_weight("c2.up")
        sess.drop_weight("c2.down")
        configs["cfg2"] = c2

    # ---- end to end through the C ABI with host buffers -----------------
    L = _lib.load()
    hostA = {K: torch.randn(M, K, generator=torch.Generator().manual_seed(K)).pin_memory()
             for K in A}
    hostY = {p.name: torch.empty(M, p.N).pin_memory() for p in projs}
    calls = [(p.name.encode(), hostA[p.K].data_ptr(), hostY[p.name].data_ptr()) for p in projs]
    h = ctypes.c_void_p(sess.handle)
    fn = L.ort_cuda_matmul_nbits

    def step_e2e():
        for nm, pa, py in calls:
            rc = fn(h, nm, pa, M, py, _lib.HOST_IO)
            if rc:
                _lib.check(rc, "ort_cuda_matmul_nbits")

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

    # ---- sharded results against one GPU (N > 1) ----------------------------
    parity = None
    if world > 1:
        parity = sharded_parity(sess, projs, weights, rank, dev, barrier)

    stats = bench.max_over_ranks([ms_step, e2e_ms, big_ms, pf_ms, pf_big_ms])
    ms_step, e2e_ms, big_ms, pf_ms, pf_big_ms = stats
    tot = torch.tensor([launches], dtype=torch.float64)
    if world > 1:
        dist.all_reduce(tot, op=dist.ReduceOp.SUM)
    launches = tot.item()

    if rank == 0:
        achieved = big_bytes / (big_ms * 1e-3) / 1e9
        traffic, traffic_note = None, None
        tp = os.path.join(ROOT, "profiles", "gemv_lm_head_traffic.json")
        if os.path.exists(tp):
            tr = json.load(open(tp)).get("plans", {})
            key = str(plans.get(big.name))
            if key in tr and world == 1:
                traffic = tr[key]
                traffic_note = f"ncu capture of the same plan ({key}), all of the op's launches"
            elif key in tr:
                # a 1-GPU capture of the full weight; a rank's shard moves its
                # share of it (the traffic grows with the columns)
                traffic = tr[key] * (bb - ba) / big.N
                traffic_note = f"1-GPU ncu capture of plan {key} scaled to this rank's shard"
            else:
                traffic_note = (f"no capture of the plan this run chose ({key}); captured: "
                                f"{sorted(tr)}")
        cpu = None
        if do_cpu:
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
            "data": "synthetic (random-init int4 weights of the named shapes, seeded)",
            "config": {"workload": "cfg5 decode step at M=1: MatMulNBits qkv 4096x6144, o "
                                   "4096x4096, gate_up 4096x28672, down 14336x4096, lm_head "
                                   "4096x128256; bits 4, block 128, fp16 scales, packed zp",
                       "mode": args.mode,
                       "gemv_plans": plans,
                       "launch": ("op-by-op calls" if args.eager else
                                  "CUDA graph of the timed steps, one replay"),
                       "parallelism": f"N-sharded x{world}" + (
                           " + Y exchanged over peer memory (the GEMV pushes its columns to "
                           "every peer)" if world > 1 else ""),
                       "l2": "inputs larger than L2 (about 387 MB of weights per step)"},
            "roofline": {"bound": "hbm",
                         "kernel": f"int4 GEMV op ({big.name}: the GEMV launch, plus the "
                                   "chunk-sum launch when its tuned plan is split-K, plus the "
                                   "landing of the peers' columns when N > 1)",
                         "timing": "event pair around the op in a second replay of the steps",
                         "achieved": achieved, "peak": hbm, "unit": "GB/s",
                         "frac": achieved / hbm, "peak_kind": hbm_kind,
                         "traffic": traffic, "traffic_source": traffic_note,
                         "bytes_per_launch": big_bytes},
            "cpu_baseline": cpu,
            "e2e": {"value": job_bytes / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": e2e_ms,
                    "call": "ort_cuda_matmul_nbits(..., ORT_CUDA_HOST_IO) on pinned host "
                            "buffers, one synchronous call per op"},
            "gpu_launches": int(launches),
            "clocks": clk,
            "prefill": {
                "value": job_flops / (pf_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                "M": PREFILL_M, "mode": "mma_f16", "ms_per_step": pf_ms, "steps": pf_steps,
                "roofline": {"bound": "tensor",
                             "kernel": f"int4 dequant + tcgen05 GEMM ({big.name})",
                             "achieved": big_flops / (pf_big_ms * 1e-3) / 1e12,
                             "peak": tpk, "unit": "TFLOP/s",
                             "frac": big_flops / (pf_big_ms * 1e-3) / 1e12 / tpk,
                             "peak_kind": tpk_kind},
            },
            "configs": configs,
        }
        if parity is not None:
            line["sharded_parity"] = parity
        print(json.dumps(line), flush=True)
    sess.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def sharded_parity(sess, projs, weights, rank, dev, barrier):
    """Every rank runs the headline ops (M=1, exact) and the prefill ops
    (M=2048, fp16 mode) on the same inputs; rank 0 also runs them on a
    single-GPU session of the full weights and compares."""
    import torch
    from onnx_runtime_dart_b200 import CudaSession, _lib
    gen = torch.Generator(device=dev).manual_seed(SEED + 9)
    pf = _lib.flags_mode(_lib.MODES["mma_f16"])
    got = {}
    for M, fl in ((1, 0), (16, 0), (PREFILL_M, pf)):
        for p in projs:
            a = torch.randn(M, p.K, device=dev, generator=gen)
            got[(M, p.name)] = (a, sess.matmul_nbits(p.name, a, flags=fl))
    barrier()
    out = None
    if rank == 0:
        one = CudaSession(dev.index)
        one.set_stream(torch.cuda.current_stream().cuda_stream)
        for p in projs:
            B, s, z = weights[p.name]
            one.upload_nbits(p.name, B, s, z, k=p.K, n=p.N, block_size=BS)
        bit = {}
        rel = 0.0
        for (M, name), (a, y) in got.items():
            ref = one.matmul_nbits(name, a, flags=pf if M == PREFILL_M else 0)
            same = bool(torch.equal(ref, y))
            if M == PREFILL_M:
                d = (ref - y).abs().max().item() / max(ref.abs().max().item(), 1e-30)
                rel = max(rel, d)
            bit.setdefault(M, True)
            bit[M] = bit[M] and same
        one.close()
        # which weights this rank keeps whole (size-based placement) and which
        # it shards
        place = {p.name: ("replicated" if sess.weight_columns(p.name) == (0, p.N) else "sharded")
                 for p in projs}
        out = {"ops": len(projs), "reference": "single-GPU session of the same weights on rank 0",
               "placement": place,
               "bitwise_m1": bit[1], "bitwise_m16": bit[16],
               "prefill_bitwise": bit[PREFILL_M], "prefill_max_rel": rel,
               "prefill_mode": "mma_f16"}
    barrier()
    return out


if __name__ == "__main__":
    main()
