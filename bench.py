"""Benchmark of the chunked FP16-accumulate GEMM (f16acc.mm) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (the configuration the headline metric is quoted
on): C = A @ B, M = N = K = 4096, A and B fp16 ~ N(0,1)/sqrt(K)*4 (seeded),
B row-major, fp16 output, chunked mode (FP16-accumulated 32-long chunks summed
in FP32, device-side flag + redo).  One step = GEMMS_PER_STEP such products,
rotating over INPUT_SETS independent (A, B) pairs whose footprint exceeds the
126 MB L2, so no step reuses L2-resident operands.

Multi-GPU (torchrun, one rank per GPU): M-sharded token batches are
independent, so every rank runs the same per-GPU work on its own inputs with no
collective on the data path ("scaling": "weak"); the time is the max over ranks.

--impl reference times the reference's CPU path (the oracle restatement of
steppergg/f16acc f16acc/kernel.py:37-81: chunked emulation) on the host cores,
rank 0 only, on a bounded row sample of the same workload.

Prints one JSON line (rank 0).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

M = N = K = 4096
GEMMS_PER_STEP = 32
INPUT_SETS = 4
METRIC = "TFLOPS @4096^3 FP16 (chunked FP16-accumulate GEMM, f16acc.mm)"
UNIT = "TFLOPS"
FALLBACK_PEAK_TFLOPS = 1590.0


def flops_per_gemm() -> float:
    return 2.0 * M * N * K


def make_inputs(torch, device, seed, sets):
    g = torch.Generator(device=device).manual_seed(seed)
    scale = 4.0 / K ** 0.5
    out = []
    for _ in range(sets):
        a = (torch.randn(M, K, device=device, generator=g) * scale).half()
        b = (torch.randn(K, N, device=device, generator=g) * scale).half()
        out.append((a, b))
    return out


def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["bf16_tflops"]), "measured (MEASURED_PEAKS.json bf16_tflops, cuBLAS bf16 burst)"
    except Exception:
        return FALLBACK_PEAK_TFLOPS, "fallback (1.59 PFLOP/s, earlier measurement on this pool)"


def profiled_traffic():
    """DRAM bytes per main-kernel launch from the committed ncu summary, or None."""
    p = os.path.join(ROOT, "profiles", "tc_gemm_chunked_4096.md")
    try:
        for line in open(p):
            if line.strip().startswith("traffic_bytes_per_launch:"):
                return int(float(line.split(":", 1)[1].strip()))
    except OSError:
        pass
    return None


# ---------------------------------------------------------------- distributed plumbing
def dist_setup(torch, want_nccl: bool):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and want_nccl:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def max_over_ranks(torch, value: float, world: int, device) -> float:
    if world == 1:
        return value
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(torch, world: int):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


# ---------------------------------------------------------------- CPU baseline (oracle)
def cpu_sample(rows: int, seed: int = 1):
    import numpy as np

    from oracle import oracle as O

    rng = np.random.default_rng(seed)
    scale = 4.0 / K ** 0.5
    a = (rng.standard_normal((rows, K)) * scale).astype(np.float16)
    b = (rng.standard_normal((K, N)) * scale).astype(np.float16)
    t0 = time.perf_counter()
    O.gemm_chunked(a, b, round_every=32)
    dt = time.perf_counter() - t0
    return dt, 2.0 * rows * N * K / dt / 1e12


def cpu_threads():
    """Give the CPU path every host thread (torchrun pins OMP_NUM_THREADS=1)
    and report the count in effect."""
    from oracle import oracle as O

    return O.set_threads(len(os.sched_getaffinity(0)) or os.cpu_count() or 1)


def cpu_baseline(target_s: float = 10.0):
    """Chunked emulation of rows of the 4096^3 product, sized to ~target_s."""
    cores = cpu_threads()
    dt, _ = cpu_sample(16)
    rows = int(max(16, min(M, 16 * target_s / max(dt, 1e-3))))
    dt, tflops = cpu_sample(rows)
    return {"value": tflops, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"oracle chunked emulation (oracle/f16acc_oracle.c, OpenMP) of {rows} of the 4096 rows "
                      f"of one 4096^3 product: {dt:.1f} s"}


# ---------------------------------------------------------------- reference arm
def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    cores = cpu_threads()
    # size each step so the whole --steps/--warmup run stays within ~2 minutes
    dt16, _ = cpu_sample(16)
    budget = 120.0 / max(1, args.steps + args.warmup)
    rows = int(max(16, min(M, 16 * budget / max(dt16, 1e-3))))
    for _ in range(args.warmup):
        cpu_sample(rows)
    times = []
    for _ in range(args.steps):
        dt, _ = cpu_sample(rows)
        times.append(dt)
    total = sum(times)
    value = args.steps * 2.0 * rows * N * K / total / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": total / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp16", "data": "synthetic",
        "config": {"workload": "config 2: 4096^3 fp16 GEMM, N(0,1)/sqrt(K)*4, chunked FP16 accumulate",
                   "rows_per_step": rows},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": f"{rows} rows of the 4096^3 product per step (reference chunked semantics, "
                                   "oracle/f16acc_oracle.c)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- our arm
def run_ours(args):
    import torch

    from f16acc_b200 import _lib
    from f16acc_b200.kernel import mm, mm_ex, plan, tile_flags, workspace_bytes
    from f16acc_b200.nvml import ClockSampler

    world, rank, local = dist_setup(torch, want_nccl=True)
    if args.gpus != world and world > 1:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = False
    stream = torch.cuda.current_stream(dev)
    variant = {v: k for k, v in _lib.VARIANT_NAMES.items()}[args.variant]

    sets = make_inputs(torch, dev, seed=1 + rank, sets=INPUT_SETS)
    outs = [torch.empty(M, N, device=dev, dtype=torch.float16) for _ in range(INPUT_SETS)]
    wss = [torch.empty(workspace_bytes(M, N, K), device=dev, dtype=torch.uint8) for _ in range(INPUT_SETS)]

    def one(i):
        # one launch: the chunked main pass with its flagged tiles redone inside the kernel
        a, b = sets[i % INPUT_SETS]
        mm_ex(a, b, torch.float16, True, variant=variant, out=outs[i % INPUT_SETS], workspace=wss[i % INPUT_SETS])

    def step():
        for i in range(GEMMS_PER_STEP):
            one(i)

    # warm-up (also loads modules / sets attributes)
    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()

    # ---- timed region: K steps, events on the launching stream, barrier + sync both sides
    clocks = ClockSampler(local)
    barrier(torch, world)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with clocks:
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        torch.cuda.synchronize()
    barrier(torch, world)
    ms = ev0.elapsed_time(ev1)
    ms_max = max_over_ranks(torch, ms, world, dev)
    gemms_total = args.steps * GEMMS_PER_STEP * world
    value = gemms_total * flops_per_gemm() / (ms_max / 1e3) / 1e12
    launches = args.steps * GEMMS_PER_STEP  # one kernel per product

    # ---- roofline: the kernel's own duration, one event pair per launch
    n_main = min(64, max(16, args.steps * 2))
    main_ms = []
    for i in range(n_main):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        one(i)
        e1.record(stream)
        main_ms.append((e0, e1))
    torch.cuda.synchronize()
    main_avg_ms = statistics.mean(e0.elapsed_time(e1) for e0, e1 in main_ms)
    peak, peak_src = measured_peak()
    achieved = flops_per_gemm() / (main_avg_ms / 1e3) / 1e12

    # ---- accuracy (config 2): max rel err vs FP64, flagged tiles
    a, b = sets[0]
    c = mm(a, b)
    ref = a.double() @ b.double()
    max_rel = ((c.double() - ref).abs().max() / ref.abs().max()).item()
    del ref
    pl = plan(a, b, variant)
    flagged = int(tile_flags(wss[0], pl).sum().item())

    # ---- cuBLAS on the same box for context (FP32 accumulate and FP16 accumulate)
    def time_torch(fn, reps=3 * GEMMS_PER_STEP):
        for i in range(8):
            fn(i)
        torch.cuda.synchronize()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        for i in range(reps):
            fn(i)
        s1.record(stream)
        torch.cuda.synchronize()
        return reps * flops_per_gemm() / (s0.elapsed_time(s1) / 1e3) / 1e12

    mmod = torch.backends.cuda.matmul
    cublas_f32 = time_torch(lambda i: torch.mm(*sets[i % INPUT_SETS], out=outs[i % INPUT_SETS]))
    mmod.allow_fp16_accumulation = True
    try:
        cublas_f16 = time_torch(lambda i: torch.mm(*sets[i % INPUT_SETS], out=outs[i % INPUT_SETS]))
    finally:
        mmod.allow_fp16_accumulation = False

    # ---- e2e through the public API with host buffers (pinned), copies inside the timed region.
    # Three streams: uploads of product i+1 and the download of product i-1 overlap product
    # i's kernel (PCIe is full duplex), as a serving loop would run them.
    e2e_steps = max(1, min(args.steps, 3))
    host_in = [(a.cpu().pin_memory(), b.cpu().pin_memory()) for a, b in sets]
    host_out = [torch.empty(M, N, dtype=torch.float16).pin_memory() for _ in range(INPUT_SETS)]
    dev_in = [(torch.empty_like(a), torch.empty_like(b)) for a, b in sets]
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def ev():
        return torch.cuda.Event()

    used = [None] * INPUT_SETS  # set j's device inputs free again (its product finished)
    torch.cuda.synchronize()
    barrier(torch, world)
    x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    x0.record(stream)
    up.wait_event(x0)
    for _ in range(e2e_steps):
        for i in range(GEMMS_PER_STEP):
            j = i % INPUT_SETS
            with torch.cuda.stream(up):
                if used[j] is not None:
                    up.wait_event(used[j])
                dev_in[j][0].copy_(host_in[j][0], non_blocking=True)
                dev_in[j][1].copy_(host_in[j][1], non_blocking=True)
                ready = ev()
                ready.record(up)
            stream.wait_event(ready)
            cj = mm(dev_in[j][0], dev_in[j][1])
            done = ev()
            done.record(stream)
            used[j] = done
            with torch.cuda.stream(down):  # downloads stay in order on this stream
                down.wait_event(done)
                host_out[j].copy_(cj, non_blocking=True)
                cj.record_stream(down)
    last = ev()
    last.record(down)
    stream.wait_event(last)
    x1.record(stream)
    torch.cuda.synchronize()
    barrier(torch, world)
    e2e_ms = max_over_ranks(torch, x0.elapsed_time(x1), world, dev)
    e2e_value = e2e_steps * GEMMS_PER_STEP * world * flops_per_gemm() / (e2e_ms / 1e3) / 1e12
    h2d = GEMMS_PER_STEP * 2 * M * K * 2
    d2h = GEMMS_PER_STEP * M * N * 2

    line = None
    if rank == 0:
        cpu = cpu_baseline() if world == 1 else None
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp16", "data": "synthetic",
            "config": {"workload": "config 2: C = A @ B, 4096^3 fp16, N(0,1)/sqrt(K)*4, B row-major, fp16 out, "
                                   "chunked FP16 accumulate, flagged tiles redone in FP32 inside the same kernel",
                       "gemms_per_step": GEMMS_PER_STEP, "per_gpu": "one 4096-row M shard per product",
                       "l2": f"inputs rotate over {INPUT_SETS} (A,B) sets = {INPUT_SETS * 64} MiB > 126 MB L2",
                       "parallelism": f"dp{world} (independent M shards, no collective)",
                       "variant": args.variant, "kernel": _lib.VARIANT_NAMES.get(pl["variant"]),
                       "tile": list(pl["tile"])},
            "max_rel_err_vs_fp64": max_rel,
            "flagged_tiles": flagged,
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "traffic": profiled_traffic(),
                         "kernel": "tc_gemm_kernel, chunked (main pass + in-kernel redo)", "main_kernel_ms": main_avg_ms,
                         "peak_source": peak_src},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "steps": e2e_steps,
                    "api": "f16acc_b200.mm with pinned host copies; uploads, kernel and download on three "
                           "streams so consecutive products overlap"},
            "gpu_launches": launches,
            "clocks": clocks.summary(),
            "context": {"cublas_f32acc_tflops": cublas_f32, "cublas_f16acc_tflops": cublas_f16,
                        "reference_published": "65.7 TFLOPS f16acc at 4096^3 on RTX 4060 Ti (README.md:29)"},
        }
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)
    return 0


def rel_err(x, ref) -> float:
    return ((x.double() - ref).abs().max() / ref.abs().max()).item()


def run_workload(args):
    """The other BASELINE configs (f16acc_b200/workloads.py): one JSON line each."""
    import torch

    from f16acc_b200 import workloads as W

    want_nccl = args.workload in ("nshard", "prefill")
    world, rank, local = dist_setup(torch, want_nccl=want_nccl)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    line = {"workload": args.workload, "n_gpus": world, "data": "synthetic"}
    if args.workload == "shapes":
        line["config"] = "config 3: Qwen2.5-1.5B linear shapes, M=2048, weight [N,K], fp16 out"
        line["results"] = W.shapes(dev)
    elif args.workload == "overflow":
        line["config"] = "config 4: 4096^3 N(0,1), 1% rows/cols x64; 4b: ~1% of tiles overflow"
        line["results"] = W.overflow(dev)
    elif args.workload == "decode":
        hbm = None
        try:
            with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
                hbm = float(json.load(f)["hbm_gbs"])
        except (OSError, KeyError, ValueError):
            pass
        line["config"] = ("few-row products (M = 1..64 decode tokens) on the Qwen2.5-1.5B weight shapes, "
                          "weight [N,K], fp16 out; CUDA-graph timing over weight copies > L2")
        line["hbm_peak_gbs"] = hbm
        line["results"] = W.decode(dev, hbm_gbs=hbm)
    elif args.workload == "nshard":
        from f16acc_b200.kernel import mm
        from f16acc_b200.shard import nshard_mm, shard_bounds

        n = args.size
        g = torch.Generator(device=dev).manual_seed(3)  # same A and B on every rank
        a = torch.randn(n, n, device=dev, generator=g).half()
        b = torch.randn(n, n, device=dev, generator=g).half()
        lo, hi = shard_bounds(n, world, rank)
        b_shard = b[:, lo:hi].contiguous()

        def step(gather=True, blocks=args.nshard_blocks, reserve=args.nshard_reserve):
            if world == 1:
                return mm(a, b_shard)
            return nshard_mm(a, b_shard, gather=gather, blocks=blocks, reserve_sms=reserve)

        def timed(fn):
            for _ in range(max(3, args.warmup)):
                fn()
            torch.cuda.synchronize()
            barrier(torch, world)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(args.steps):
                r = fn()
            e1.record()
            torch.cuda.synchronize()
            barrier(torch, world)
            return max_over_ranks(torch, e0.elapsed_time(e1) / args.steps, world, dev), r

        times = {}
        times["compute_only"], c = timed(lambda: step(False))
        times["with_allgather"], c = timed(lambda: step(True))
        if world > 1:
            from f16acc_b200.shard import nshard_mm_fused

            times["fused_gemm_allgather"], c = timed(lambda: nshard_mm_fused(a, b_shard))
        if world > 1 and args.nshard_sweep:
            import torch.distributed as dist

            panel = torch.empty(n, hi - lo, dtype=torch.float16, device=dev)
            flat = torch.empty(world * n, hi - lo, dtype=torch.float16, device=dev)
            t_ag, _ = timed(lambda: dist.all_gather_into_tensor(flat, panel))
            times["allgather_only"] = t_ag
            line["allgather_bus_gbs"] = (world - 1) * panel.numel() * 2 / (t_ag / 1e3) / 1e9
            for blocks in (1, 2, 8):
                for reserve in (0, 16):
                    times[f"with_allgather_blocks{blocks}_reserve{reserve}"], _ = timed(
                        lambda: step(True, blocks, reserve))
        # the (gathered) C is the full product: check the first 64 rows against FP64
        ref = a[:64].double() @ b.double()
        line["max_rel_err_first_64_rows"] = max_over_ranks(torch, rel_err(c[:64], ref), world, dev)
        del ref
        line["config"] = f"config 4c: N-sharded {n}^3 fp16 over {world} ranks, NCCL all-gather of C"
        flops = 2.0 * n ** 3
        line["results"] = {k: {"ms": v, "tflops": flops / v / 1e9} for k, v in times.items()}
        line["scaling"] = "strong"
    elif args.workload == "prefill":
        r = W.prefill(dev, rank=rank, world=world)
        ms_c = max_over_ranks(torch, r["ms_cublas"], world, dev)
        ms_f = max_over_ranks(torch, r["ms_f16acc"], world, dev)
        tokens = 8 * 2048
        line["config"] = ("config 5: random-init Qwen2.5-1.5B architecture (28 layers, hidden 1536, 12/2 heads, "
                          "intermediate 8960, vocab 151936, tied), 8 prompts x 2048 tokens, data parallel")
        line["results"] = {"tokens_per_s_f16acc": tokens / (ms_f / 1e3), "tokens_per_s_cublas": tokens / (ms_c / 1e3),
                           "speedup": ms_c / ms_f, "top1_agreement_rank0": r["top1_agreement"],
                           "routed_calls_per_pass_rank0": r["routed_calls_per_pass"]}
        line["scaling"] = "strong"
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def main(argv=None):
    ap = argparse.ArgumentParser(description="f16acc B200 benchmark")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--variant", choices=["auto", "tcgen05", "mma_sync"], default="auto")
    ap.add_argument("--workload", choices=["gemm4096", "shapes", "overflow", "nshard", "prefill", "decode"],
                    default="gemm4096",
                    help="gemm4096 is the headline line; the others print their own JSON line")
    ap.add_argument("--size", type=int, default=16384, help="matrix size for --workload nshard")
    ap.add_argument("--nshard-blocks", type=int, default=4, help="row blocks the sharded gather is pipelined in")
    ap.add_argument("--nshard-reserve", type=int, default=16, help="SMs left free for NCCL during the product")
    ap.add_argument("--nshard-sweep", action="store_true", help="also time the bare all-gather and other blockings")
    args = ap.parse_args(argv)
    if args.impl == "reference":
        return run_reference(args)
    if args.workload != "gemm4096":
        return run_workload(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
