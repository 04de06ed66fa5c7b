"""N-sharded sessions on two GPUs (skipped with fewer).

Each rank keeps its column shard of every weight and all-gathers Y: over
peer memory (both ranks' exchange buffers mapped with CUDA IPC) when the
slices fit, else with NCCL.  Two spawned processes, one per GPU, check the
sharded results against the oracle, a prefill-sized output that takes the
NCCL path, and a CUDA-graph replay of sharded calls against eager calls.
These sessions shard every weight (replicate bytes 0); a weight below the
size-based placement threshold is then kept whole on every rank and must
give the single-GPU bits with no exchange.
"""
import datetime
import multiprocessing as mp
import os
import socket
import traceback

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = pytest.mark.gpu
WORLD = 2


def _gpus():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _entry(rank, port, q):
    import sys
    sys.path.insert(0, ROOT)
    try:
        q.put((rank, True, _rank_main(rank, port)))
    except Exception:
        q.put((rank, False, traceback.format_exc()))


def _rank_main(rank, port):
    import torch
    import torch.distributed as dist
    from oracle import oracle as O
    from onnx_runtime_dart_b200 import CudaSession, _lib
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=WORLD, timeout=datetime.timedelta(seconds=60))
    try:
        obj = [CudaSession.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        s = CudaSession(rank, rank=rank, world=WORLD, nccl_id=obj[0], timeout_ms=30000)
        s.set_replicate_bytes(0)  # every weight sharded: the exchange paths under test
        st = torch.cuda.Stream()
        s.set_stream(st.cuda_stream)
        out = {}
        rng = np.random.default_rng(9)  # the same weights and inputs on every rank
        shapes = {"tm": (1024, 50000, 32), "sk": (4096, 3000, 128), "pf": (1024, 8192, 64)}
        W = {}
        for name, (K, N, bs) in shapes.items():
            B, sc, z = O.make_nbits_weight(rng, K, N, bs, zero_points=True)
            s.upload_nbits(name, B, sc, z, k=K, n=N, block_size=bs)
            W[name] = (B, sc, z, K, N, bs)
        # a dense weight: its sharded Gemm exchanges Y by peer loads (pull),
        # interleaved below with the GEMV's pushes (both advance one epoch)
        Wd = rng.standard_normal((256, 640)).astype(np.float32)
        s.upload_dense("d", Wd, trans_b=False)
        # decode: exact mode against the oracle, and bit for bit against a
        # single-GPU session (rank 0): M <= 8 pushes from one GEMV pass, M = 16
        # from two passes of 8 rows
        got = {}
        for name in ("tm", "sk"):
            B, sc, z, K, N, bs = W[name]
            for M in (1, 3, 16):
                A = rng.standard_normal((M, K)).astype(np.float32)
                y = s.matmul_nbits(name, A)
                yd = s.gemm("d", rng.standard_normal((M, 256)).astype(np.float32))
                ref = O.matmul_nbits(A, B, sc, z, K, N, 4, bs, threads=8)
                out[f"{name}{M}"] = float(np.abs(y - ref).max() / np.abs(ref).max())
                got[(name, M)] = (A, y)
                got[("d", M)] = yd
        # size-based placement: a weight below the threshold kept whole on
        # every rank, computed there (interleaved with sharded calls)
        s.set_replicate_bytes(-1)
        Br, scr, zr = O.make_nbits_weight(rng, 2048, 3000, 128, zero_points=True)
        s.upload_nbits("rep", Br, scr, zr, k=2048, n=3000, block_size=128)
        s.set_replicate_bytes(0)
        for M in (1, 16, 300):
            A = rng.standard_normal((M, 2048)).astype(np.float32)
            got[("rep", M)] = (A, s.matmul_nbits("rep", A))
            s.matmul_nbits("sk", rng.standard_normal((M, 4096)).astype(np.float32))
        if rank == 0:
            one = CudaSession(rank)
            for name in ("tm", "sk"):
                B, sc, z, K, N, bs = W[name]
                one.upload_nbits(name, B, sc, z, k=K, n=N, block_size=bs)
                for M in (1, 3, 16):
                    A, y = got[(name, M)]
                    out[f"bitwise_{name}{M}"] = bool(np.array_equal(one.matmul_nbits(name, A), y))
            one.upload_nbits("rep", Br, scr, zr, k=2048, n=3000, block_size=128)
            for M in (1, 16, 300):
                A, y = got[("rep", M)]
                out[f"bitwise_rep{M}"] = bool(np.array_equal(one.matmul_nbits("rep", A), y))
            one.close()
        # prefill-sized output (4096 x 4096 floats per rank): NCCL path
        B, sc, z, K, N, bs = W["pf"]
        A = rng.standard_normal((4096, K)).astype(np.float32)
        y = s.matmul_nbits("pf", A, flags=_lib.flags_mode(_lib.MODES["mma_f16"]))
        ref = O.matmul_nbits(A[:64], B, sc, z, K, N, 4, bs, threads=8)
        out["pf"] = float(np.abs(y[:64] - ref).max() / np.abs(ref).max())
        # graph replay of sharded calls equals eager calls bit for bit
        with torch.cuda.stream(st):
            x = torch.empty(1, 4096, device="cuda")
            h = torch.empty(1, 3000, device="cuda")
            g = torch.empty(1, 50000, device="cuda")
            xs = torch.empty(1, 1024, device="cuda")

            def run():
                s.matmul_nbits("sk", x, out=h)
                s.matmul_nbits("tm", xs, out=g)

            x.copy_(torch.randn(1, 4096, generator=torch.Generator().manual_seed(1)))
            xs.copy_(torch.randn(1, 1024, generator=torch.Generator().manual_seed(2)))
            run()
            st.synchronize()
            s.graph_begin()
            run()
            gid = s.graph_end()
            same = True
            for seed in (3, 4):
                x.copy_(torch.randn(1, 4096, generator=torch.Generator().manual_seed(seed)))
                xs.copy_(torch.randn(1, 1024, generator=torch.Generator().manual_seed(seed + 10)))
                run()
                st.synchronize()
                eh, eg = h.clone(), g.clone()
                s.graph_launch(gid)
                st.synchronize()
                same = same and torch.equal(eh, h) and torch.equal(eg, g)
            s.graph_drop(gid)
        out["graph_same"] = bool(same)
        s.sync()
        s.close()
        return out
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(_gpus() < WORLD, reason="needs two GPUs")
def test_two_gpu_sharded_results():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_entry, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(WORLD):
            r, ok, val = q.get(timeout=300)
            res[r] = (ok, val)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r in range(WORLD):
        ok, val = res[r]
        assert ok, val
        for key in ("tm1", "tm3", "tm16", "sk1", "sk3", "sk16"):
            assert val[key] <= 1e-5, (r, key, val[key])
        if r == 0:
            for key in ("tm1", "tm3", "tm16", "sk1", "sk3", "sk16", "rep1", "rep16", "rep300"):
                assert val["bitwise_" + key], key
        assert val["pf"] <= 2e-3, (r, val["pf"])
        assert val["graph_same"], r


def _timeout_entry(rank, port, q):
    import sys
    sys.path.insert(0, ROOT)
    try:
        q.put((rank, True, _timeout_main(rank, port)))
    except Exception:
        q.put((rank, False, traceback.format_exc()))


def _timeout_main(rank, port):
    """Rank 1 skips an operation: rank 0's wait for its columns runs out
    after the session's (short) peer-wait bound, the kernel returns, the
    next synchronising call reports ORT_CUDA_ERR_TIMEOUT, and both sessions
    still close.  The failure is made on the host (a rank that does not
    call); nothing faults or hangs on the GPU."""
    import torch
    import torch.distributed as dist
    from oracle import oracle as O
    from onnx_runtime_dart_b200 import CudaSession, StateError, _lib
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=WORLD, timeout=datetime.timedelta(seconds=60))
    try:
        obj = [CudaSession.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        s = CudaSession(rank, rank=rank, world=WORLD, nccl_id=obj[0], timeout_ms=30000)
        s.set_replicate_bytes(0)  # sharded: the op has an exchange to wait in
        s.set_peer_wait(50)
        rng = np.random.default_rng(3)
        K, N = 1024, 4096
        B, sc, z = O.make_nbits_weight(rng, K, N, 128, zero_points=True)
        s.upload_nbits("w", B, sc, z, k=K, n=N, block_size=128)
        a = torch.randn(1, K, device="cuda")
        y = s.matmul_nbits("w", a)  # together: plans timed, exchange completes
        s.sync()
        out = {"first_ok": bool(torch.isfinite(y).all())}
        dist.barrier()
        if rank == 0:
            s.matmul_nbits("w", a)  # rank 1 never takes part
            try:
                s.sync()
                out["timeout"] = None
            except StateError as e:
                out["timeout"] = e.code if hasattr(e, "code") else str(e)
                out["msg"] = str(e)
        dist.barrier()
        s.close()
        out["closed"] = True
        return out
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(_gpus() < WORLD, reason="needs two GPUs")
def test_two_gpu_peer_wait_expires():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_timeout_entry, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(WORLD):
            r, ok, val = q.get(timeout=300)
            res[r] = (ok, val)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r in range(WORLD):
        ok, val = res[r]
        assert ok, val
        assert val["first_ok"] and val["closed"], (r, val)
    from onnx_runtime_dart_b200 import _lib
    assert res[0][1]["timeout"] == _lib.ERR_TIMEOUT, res[0][1]
