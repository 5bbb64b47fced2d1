"""Multi-rank partitioning logic on CPU ranks (gloo, world size 2): N-column
shards with the pipelined all-gather, and independent M-row shards.  The
per-rank product is a float64 CPU matmul standing in for the GPU kernel, so
only the partition / exchange / placement logic is under test here; the GPU
kernel itself is covered by the -m gpu tests."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from f16acc_b200.shard import mshard_rows, nshard_mm, shard_bounds


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _cpu_mm(a, b, out_dtype):
    return (a.double() @ b.double()).to(out_dtype)


def _worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(0)
        M, K, N = 37, 24, 8 * world
        a = torch.randn(M, K, generator=g).half()
        b = torch.randn(K, N, generator=g).half()
        lo, hi = shard_bounds(N, world, rank)
        full = nshard_mm(a, b[:, lo:hi], mm_fn=_cpu_mm, out_dtype=torch.float32, blocks=3)
        blocked = nshard_mm(a, b[:, lo:hi], mm_fn=_cpu_mm, out_dtype=torch.float32, blocks=2, row_major=False)
        local = nshard_mm(a, b[:, lo:hi], mm_fn=_cpu_mm, out_dtype=torch.float32, gather=False)
        ref = (a.double() @ b.double()).float()
        ok_full = torch.equal(full, ref)
        ok_blocked = all(torch.equal(blocked[p], ref[:, shard_bounds(N, world, p)[0]:shard_bounds(N, world, p)[1]])
                         for p in range(world))
        ok_local = torch.equal(local, ref[:, lo:hi])
        rows = mshard_rows(a, rank, world)
        r0, r1 = shard_bounds(M, world, rank)
        ok_rows = torch.equal(rows, a[r0:r1])
        results[rank] = (ok_full, ok_blocked, ok_local, ok_rows)
    finally:
        dist.destroy_process_group()


def test_shard_bounds_cover_exactly():
    for n in (0, 1, 7, 64, 100):
        for p in (1, 2, 3, 8):
            spans = [shard_bounds(n, p, i) for i in range(p)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[i][1] == spans[i + 1][0] for i in range(p - 1))
            assert max(h - l for l, h in spans) - min(h - l for l, h in spans) <= 1
    with pytest.raises(ValueError):
        shard_bounds(4, 2, 2)


def test_nshard_gather_and_mshard_two_ranks():
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        results = mgr.dict()
        procs = [ctx.Process(target=_worker, args=(r, world, port, results)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
            assert p.exitcode == 0
        for r in range(world):
            assert results[r] == (True, True, True, True), (r, results[r])
