"""Multi-GPU partitioning of the chunked GEMM (one process per GPU).

Two ways the product shards across the GPUs of one node:

* N-column shards (`nshard_mm`): rank r holds A in full and the column slice
  B[:, r*N/P:(r+1)*N/P], computes its C panel with `f16acc.mm` (chunked
  accumulation, flags and redo are all local to the rank), and, only when the
  consumer needs the full matrix, the panels are all-gathered over NCCL.  The
  gather is pipelined by row blocks on a side stream so it overlaps the next
  block's compute; the gathered buffer is [P, M, N/P] (rank-blocked) and is
  either returned as is or permuted into row-major [M, N] on the device.
* N-column shards, fused (`nshard_mm_fused`): the GEMM kernel itself stores
  every finished tile into all ranks' row-major outputs over NVLink (peer
  memory from torch symmetric memory), so the exchange overlaps the math tile
  by tile and needs no SMs of its own; a device barrier ends the call.
* M-row shards (`mshard_rows`): token batches are independent, so each rank
  takes a contiguous block of rows and needs no collective at all.

The reference has no multi-GPU path (it is single-GPU Triton); this module is
new.  Every rank issues the same collectives in the same order.
"""

from __future__ import annotations

import ctypes
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


_SYMM = {}  # (M, N, dtype, device index, group name) -> (buffer, handle)


def _symmetric_output(M, N, dtype, device, group):
    """A row-major [M, N] buffer allocated on every rank of `group` with the
    other ranks' copies mapped into this process (torch symmetric memory,
    CUDA backend: plain peer mappings, no NVSHMEM).  Cached per shape."""
    import torch.distributed._symmetric_memory as symm_mem

    pg = group if group is not None else dist.group.WORLD
    key = (M, N, dtype, device.index, pg.group_name)
    hit = _SYMM.get(key)
    if hit is None:
        if symm_mem.get_backend(device) is None:
            symm_mem.set_backend("CUDA")
        buf = symm_mem.empty(M, N, dtype=dtype, device=device)
        hdl = symm_mem.rendezvous(buf, pg)
        hit = _SYMM[key] = (buf, hdl)
    return hit


def nshard_mm_fused(a: torch.Tensor, b_shard: torch.Tensor, *, out_dtype=torch.float16, chunked: bool = True,
                    group=None) -> torch.Tensor:
    """C = A @ B with B column-sharded, gathered by the GEMM itself.

    One kernel per rank computes its [M, N/P] panel and, tile by tile as the
    product runs, stores every finished tile both into its own full [M, N]
    output and into every other rank's (peer memory over NVLink,
    `f16acc_gemm_allgather`); a device-side barrier across the ranks then
    makes the gathered C complete everywhere.  Returns this rank's full
    row-major C.  The buffer is reused across calls with the same shape:
    consume (or copy) it before the next call.
    """
    from . import _lib
    from .kernel import _OUT_CODES, _check, _raise, workspace_bytes

    _check(a, b_shard)
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    M, K = a.shape
    n_local = b_shard.shape[1]
    N = world * n_local
    buf, hdl = _symmetric_output(M, N, out_dtype, a.device, group)
    esize = buf.element_size()
    order = [rank] + [r for r in range(world) if r != rank]  # own block first
    ptrs = [hdl.buffer_ptrs[r] + rank * n_local * esize for r in order]
    outs = (ctypes.c_void_p * world)(*ptrs)
    ws = torch.empty(workspace_bytes(M, n_local, K), dtype=torch.uint8, device=a.device) if chunked else None
    lib = _lib.load()
    hdl.barrier()  # no rank still reads its buffer from the previous call when the stores start
    rc = lib.f16acc_gemm_allgather(a.data_ptr(), a.stride(0), a.stride(1), b_shard.data_ptr(), b_shard.stride(0),
                                   b_shard.stride(1), outs, world, N, 1, _OUT_CODES[out_dtype], M, n_local, K,
                                   1 if chunked else 0, ws.data_ptr() if ws is not None else None,
                                   ws.numel() if ws is not None else 0, a.device.index,
                                   torch.cuda.current_stream(a.device).cuda_stream)
    if rc != _lib.OK:
        _raise(rc)
    hdl.barrier()  # every rank's tiles have landed in every buffer
    return buf


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
