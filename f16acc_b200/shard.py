"""Multi-GPU partitioning of the chunked GEMM (one process per GPU).

Two ways the product shards across the GPUs of one node:

* N-column shards (`nshard_mm`): rank r holds A in full and the column slice
  B[:, r*N/P:(r+1)*N/P], computes its C panel with `f16acc.mm` (chunked
  accumulation, flags and redo are all local to the rank), and, only when the
  consumer needs the full matrix, the panels are all-gathered over NCCL.  The
  gather is pipelined by row blocks on a side stream so it overlaps the next
  block's compute; the gathered buffer is [P, M, N/P] (rank-blocked) and is
  either returned as is or permuted into row-major [M, N] on the device.
* M-row shards (`mshard_rows`): token batches are independent, so each rank
  takes a contiguous block of rows and needs no collective at all.

The reference has no multi-GPU path (it is single-GPU Triton); this module is
new.  Every rank issues the same collectives in the same order.
"""

from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist


def shard_bounds(n: int, parts: int, index: int) -> tuple[int, int]:
    """[lo, hi) of shard `index` when n items split into `parts` near-equal shards."""
    if parts <= 0 or not (0 <= index < parts):
        raise ValueError("bad shard index")
    base, extra = divmod(n, parts)
    lo = index * base + min(index, extra)
    return lo, lo + base + (1 if index < extra else 0)


def mshard_rows(x: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """This rank's contiguous block of rows (independent token batches)."""
    lo, hi = shard_bounds(x.shape[0], world, rank)
    return x[lo:hi]


def _default_mm(a, b, out_dtype):
    from .kernel import mm

    return mm(a, b, out_dtype)


def nshard_mm(a: torch.Tensor, b_shard: torch.Tensor, *, gather: bool = True, row_major: bool = True,
              out_dtype=torch.float16, blocks: int = 4, group=None,
              mm_fn: Optional[Callable] = None, comm_stream: Optional[torch.cuda.Stream] = None,
              reserve_sms: int = 16):
    """C = A @ B with B column-sharded across the ranks of `group`.

    Every rank passes the full A [M, K] and its own B column slice [K, N/P]
    (equal widths on every rank).  Returns this rank's panel [M, N/P] when
    `gather` is False; otherwise all panels, either rank-blocked [P, M, N/P]
    (`row_major=False`) or as row-major [M, N].  The gather runs per row block
    (`blocks` of them) so block i's exchange overlaps block i+1's compute.
    `mm_fn(a, b, out_dtype)` defaults to the chunked kernel; while it runs
    with gathers in flight, the kernel is capped to all but `reserve_sms` SMs
    (the GEMM is persistent, one CTA per SM, and would otherwise keep NCCL's
    kernels from being scheduled until it finished).
    """
    default_kernel = mm_fn is None
    mm_fn = mm_fn or _default_mm
    M = a.shape[0]
    n_local = b_shard.shape[1]
    if not gather:
        return mm_fn(a, b_shard, out_dtype)
    world = dist.get_world_size(group)
    width = torch.tensor([n_local], dtype=torch.int64, device=a.device if a.is_cuda else "cpu")
    lo_hi = [torch.zeros_like(width) for _ in range(world)]
    dist.all_gather(lo_hi, width, group=group)
    if any(int(w.item()) != n_local for w in lo_hi):
        raise ValueError("nshard_mm needs the same shard width on every rank")
    if row_major:
        out = torch.empty(M, world * n_local, dtype=out_dtype, device=a.device)
    else:
        out = torch.empty(world, M, n_local, dtype=out_dtype, device=a.device)
    blocks = max(1, min(blocks, M))
    use_streams = a.is_cuda and torch.cuda.is_available()
    if use_streams:
        compute = torch.cuda.current_stream(a.device)
        comm = comm_stream or torch.cuda.Stream(device=a.device)

    def exchange(panel, r0, r1):
        # [P, rows, N/P] from every rank, then placed: row-major rows r0:r1 hold
        # the P panels side by side; rank-blocked keeps them stacked.
        flat = torch.empty(world * (r1 - r0), n_local, dtype=out_dtype, device=a.device)
        dist.all_gather_into_tensor(flat, panel, group=group)  # rank p's rows at [p*rows, (p+1)*rows)
        recv = flat.view(world, r1 - r0, n_local)
        if row_major:
            out[r0:r1].view(r1 - r0, world, n_local).copy_(recv.permute(1, 0, 2))
        else:
            out[:, r0:r1].copy_(recv)
        return recv

    lib = None
    if use_streams and default_kernel and reserve_sms > 0:
        from . import _lib

        lib = _lib.load()
        sms = torch.cuda.get_device_properties(a.device).multi_processor_count
        prev_limit = lib.f16acc_set_sm_limit(max(1, sms - reserve_sms))
    try:
        for i in range(blocks):
            r0, r1 = shard_bounds(M, blocks, i)
            panel = mm_fn(a[r0:r1], b_shard, out_dtype).contiguous()
            if use_streams:
                ev = torch.cuda.Event()
                ev.record(compute)
                comm.wait_event(ev)
                with torch.cuda.stream(comm):
                    recv = exchange(panel, r0, r1)
                # buffers made on the compute stream and used on comm stay allocated until comm is done
                panel.record_stream(comm)
                recv.record_stream(comm)
            else:
                exchange(panel, r0, r1)
    finally:
        if lib is not None:
            lib.f16acc_set_sm_limit(prev_limit)
    if use_streams:
        done = torch.cuda.Event()
        done.record(comm)
        compute.wait_event(done)
        out.record_stream(comm)
    return out
