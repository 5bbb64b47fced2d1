"""N-column-sharded product on 2 GPUs (needs at least 2 CUDA devices; skipped
otherwise): the fused GEMM + all-gather kernel (peer stores over NVLink) and
the NCCL-gathered path give the same full C, and it matches FP64.

Runs as 2 spawned processes, one per GPU, NCCL process group with a short
timeout; nothing here kills a rank or injects a fault."""

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, results):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from f16acc_b200.shard import nshard_mm, nshard_mm_fused, shard_bounds

        g = torch.Generator(device=dev).manual_seed(7)
        M, K, N = 1024, 768, 512 * world
        a = torch.randn(M, K, device=dev, generator=g).half()
        b = torch.randn(K, N, device=dev, generator=g).half()
        b[:, 5] *= 300.0  # one column band overflows FP16 chunks: flags + redo across peers
        a[17] *= 300.0
        lo, hi = shard_bounds(N, world, rank)
        bs = b[:, lo:hi].contiguous()
        fused = nshard_mm_fused(a, bs).clone()
        fused2 = nshard_mm_fused(a, bs).clone()  # the buffer is reused: second call, same result
        nccl = nshard_mm(a, bs)
        torch.cuda.synchronize()
        ref = a.double() @ b.double()
        fits = ref.abs() < 65000  # an fp16 store of a larger product is inf, as in the reference's cast
        err = ((fused.double()[fits] - ref[fits]).abs().max() / ref.abs().max()).item()
        results[rank] = (bool(torch.equal(fused, nccl)), bool(torch.equal(fused, fused2)), err,
                         bool(torch.isfinite(fused[fits]).all() and not torch.isnan(fused).any()))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fused_allgather_matches_nccl_gather_and_fp64():
    import torch.multiprocessing as mp

    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        results = mgr.dict()
        procs = [ctx.Process(target=_worker, args=(r, world, port, results)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=300)
            assert p.exitcode == 0
        for r in range(world):
            same_as_nccl, repeatable, err, finite = results[r]
            assert same_as_nccl and repeatable and finite
            assert err < 1e-3, err
