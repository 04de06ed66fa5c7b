"""N-sharding across ranks, on CPU with the gloo backend (world size 2).

The reference's GemmPool splits a matmul's output columns over isolates
(parallel_pool.dart:121-205) and asserts that the split never changes a bit
(parallel_pool_test.dart).  The B200 build shards the same way across GPUs:
rank r keeps columns shard_range(N, r, world) of every weight, computes its
slice and all-gathers Y.  These tests run two real processes that exchange
data through torch.distributed (gloo, 127.0.0.1), with the oracle standing in
for the device kernels: the column split covers N exactly, per-rank results
gathered over the process group equal the unsharded result bit for bit, and
a rank that fails before a collective turns into an error on the other rank
within the group's timeout instead of a hang.
"""
import datetime
import multiprocessing as mp
import os
import socket
import traceback

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(target, *args, timeout=120):
    """Runs target(rank, world, port, q, *args) in WORLD spawned processes and
    returns each rank's (ok, value) result."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_entry, args=(target, r, WORLD, port, q) + args)
             for r in range(WORLD)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(WORLD):
            r, ok, val = q.get(timeout=timeout)
            res[r] = (ok, val)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    return res


def _entry(target, rank, world, port, q, *args):
    import sys
    sys.path.insert(0, ROOT)
    try:
        q.put((rank, True, target(rank, world, port, *args)))
    except Exception:  # reported to the parent, which asserts on it
        q.put((rank, False, traceback.format_exc()))


def _init(rank, world, port, seconds=60):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=seconds))
    return dist


def _cover(rank, world, port):
    from onnx_runtime_dart_b200.workloads import shard_range
    dist = _init(rank, world, port)
    try:
        out = [None] * world
        mine = {N: shard_range(N, rank, world) for N in (1, 3, 4, 5, 1000, 1001, 4096, 128256)}
        dist.all_gather_object(out, mine)
        return out
    finally:
        dist.destroy_process_group()


def _sharded_matmul(rank, world, port, K, N, bs, M):
    import torch
    from oracle import oracle as O
    from onnx_runtime_dart_b200.workloads import (make_nbits_weight, nbits_column_shard,
                                                  shard_range)
    dist = _init(rank, world, port)
    try:
        rng = np.random.default_rng(123)          # every rank builds the same weight
        B, s, z = make_nbits_weight(rng, K, N, bs, zero_points=True)
        A = rng.standard_normal((M, K)).astype(np.float32)
        a, b = shard_range(N, rank, world)
        Bs, ss, zs = nbits_column_shard(B, s, z, K, N, bs, a, b)
        y = O.matmul_nbits(A, Bs, ss, zs, K, b - a, 4, bs) if b > a else np.zeros((M, 0), np.float32)
        # all-gather of the column slices (padded to the common shard width)
        per = shard_range(N, 0, world)[1]
        buf = torch.zeros(M, per)
        buf[:, :b - a] = torch.from_numpy(y)
        parts = [torch.zeros(M, per) for _ in range(world)]
        dist.all_gather(parts, buf)
        full = np.concatenate([p[:, :shard_range(N, r, world)[1] - shard_range(N, r, world)[0]].numpy()
                               for r, p in enumerate(parts)], axis=1)
        ref = O.matmul_nbits(A, B, s, z, K, N, 4, bs)
        return bool(np.array_equal(full, ref)), float(np.abs(full - ref).max())
    finally:
        dist.destroy_process_group()


def _one_rank_fails(rank, world, port):
    import torch
    dist = _init(rank, world, port, seconds=5)
    if rank == 1:
        raise RuntimeError("rank 1 fails before the collective")
    t = torch.ones(4)
    try:
        dist.all_reduce(t)
    except Exception as e:  # the expected outcome: an error, not a hang
        return type(e).__name__
    return "completed"


def test_shard_ranges_cover_columns_exactly():
    res = _run(_cover)
    assert all(ok for ok, _ in res.values()), res
    per_rank = res[0][1]              # every rank's ranges, gathered on rank 0
    assert res[1][1] == per_rank      # and identically on rank 1
    for N in per_rank[0]:
        ranges = [per_rank[r][N] for r in range(WORLD)]
        covered = np.zeros(N, np.int32)
        for a, b in ranges:
            assert 0 <= a <= b <= N
            assert a % 4 == 0 or a == b  # non-empty shards start on 4-column boundaries
            covered[a:b] += 1
        assert (covered == 1).all(), (N, ranges)


@pytest.mark.parametrize("K,N,bs,M", [(1024, 1000, 32, 3), (512, 130, 128, 2)])
def test_sharded_columns_allgather_bitwise(K, N, bs, M):
    res = _run(_sharded_matmul, K, N, bs, M)
    for r in range(WORLD):
        ok, val = res[r]
        assert ok, val
        equal, diff = val
        assert equal, f"rank {r}: sharded result differs from the full one by {diff}"


def test_rank_failure_is_an_error_not_a_hang():
    res = _run(_one_rank_fails, timeout=90)
    ok0, val0 = res[0]
    assert ok0, val0
    assert val0 != "completed"
    ok1, val1 = res[1]
    assert not ok1 and "rank 1 fails" in val1
