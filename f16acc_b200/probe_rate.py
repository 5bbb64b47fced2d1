"""B200 raw-rate probes (counterpart of the reference's bench/rate.py and
bench/chunkrate.py): tcgen05 MMA throughput with an FP16 vs FP32 accumulator,
and the ceiling of the chunked pipeline (MMA + per-chunk TMEM load + FP32 add)
with no global-memory traffic.

    python -m f16acc_b200.probe_rate [--chunks 4096] [--reps 5]

Prints one JSON line per probe: TFLOPS (2*128*128*32 flops per chunk per CTA)
and the fraction of the clock-normalised dense peak 148 SMs x 8192 flop/clk x
the SM clock NVML reports during the run.
"""

from __future__ import annotations

import argparse
import json
import statistics
import sys

import torch

from . import _lib
from .nvml import ClockSampler


def run(mode: int, epi_split: int, chunks: int, reps: int, dev: torch.device):
    lib = _lib.load()
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    threads = 64 + 128 * epi_split
    out = torch.empty(sms * threads, device=dev)
    stream = torch.cuda.current_stream(dev)

    def launch():
        rc = lib.f16acc_probe_chunk_rate(mode, epi_split, chunks, sms, out.data_ptr(), dev.index, stream.cuda_stream)
        if rc != 0:
            raise RuntimeError(_lib.strerror(rc))

    for _ in range(2):
        launch()
    torch.cuda.synchronize()
    ms = []
    with ClockSampler(dev.index or 0, period_s=0.002) as clocks:
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            launch()
            e1.record(stream)
            torch.cuda.synchronize()
            ms.append(e0.elapsed_time(e1))
    med = statistics.median(ms)
    flops = sms * chunks * 2.0 * 128 * 128 * 32
    return sms, med, flops / (med / 1e3) / 1e12, clocks.summary()


def trace(dev: torch.device, npairs: int = 2048) -> int:
    """The timed pair hand-off: median SM cycles of each step per pair (pairs
    npairs/10 .. 9*npairs/10 of CTA 0, all 148 CTAs running)."""
    lib = _lib.load()
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    names = ("pipeline", "pipeline_without_adds", "mma_warp_alone", "pipeline_two_mma_threads",
             "pipeline_two_mma_threads_issuer_first")
    for epi in (4, 2):
        for variant in (0, 1, 2, 3, 4):
            ev = torch.zeros(npairs * 9, dtype=torch.int64, device=dev)
            out = torch.empty(sms * (64 + 128 * epi), device=dev)
            for _ in range(3):  # the last run's stamps are read
                rc = lib.f16acc_probe_pair_trace(variant, epi, npairs, sms, ev.data_ptr(), out.data_ptr(),
                                                 dev.index or 0, torch.cuda.current_stream(dev).cuda_stream)
                if rc != 0:
                    raise RuntimeError(_lib.strerror(rc))
            torch.cuda.synchronize()
            e = ev.view(npairs, 9).cpu().tolist()
            rows = range(npairs // 10, npairs * 9 // 10)
            med = lambda f: statistics.median(f(i) for i in rows)  # noqa: E731
            res = {"probe": "pair_trace_" + names[variant], "epilogue_warps": 4 * epi,
                   "pair_period": med(lambda i: e[i + 1][4] - e[i][4]),
                   "mma_fence": med(lambda i: e[i][1] - e[i][0]),
                   "mma_first_issue": med(lambda i: e[i][2] - e[i][1]),
                   "mma_next_three_issue": med(lambda i: e[i][3] - e[i][2]),
                   "mma_commit_issue": med(lambda i: e[i][4] - e[i][3])}
            if variant != 2:
                last = lambda i: max(e[i][6], e[i][8])  # noqa: E731
                res.update({"commit_to_epilogue_wake": med(lambda i: e[i][5] - e[i][4]),
                            "epilogue_wake_to_release": med(lambda i: e[i][6] - e[i][5]),
                            "release_to_mma_wake": med(lambda i: e[i + 2][0] - last(i) if i + 2 < npairs else 0)})
            res["frac_of_peak"] = 256.0 / res["pair_period"]  # 4 MMAs of 64 cycles per pair
            print(json.dumps(res), flush=True)
    return 0


def latency(dev: torch.device, chunks: int, reps: int) -> int:
    """One thread per SM: a dependent MMA group + commit + mbarrier wait per
    iteration (suspending or spinning waits), and a two-thread mbarrier
    ping-pong; cycles per iteration at the sampled SM clock."""
    lat = [("latency_2mma_n128", 8), ("latency_1mma_n128", 9), ("latency_2mma_n64", 10), ("latency_8mma_n128", 11),
           ("latency_1mma_n128_spin", 47), ("latency_commit_only", 48), ("latency_commit_only_spin", 49),
           ("latency_2mma_n128_spin", 50), ("latency_pingpong_2hops", 51), ("latency_pingpong_2hops_spin", 52)]
    lat += [("roundtrip_16warps_mbarriers", 53), ("roundtrip_16warps_smem_flags", 54),
            ("roundtrip_16warps_named_barriers", 55), ("roundtrip_16warps_mbarrier_out_named_back", 56)]
    iters = max(256, chunks // 16)
    for name, mode in lat:
        sms, ms, _, clk = run(mode, 4 if mode >= 53 else 2, iters, reps, dev)
        ns = ms * 1e6 / iters
        mhz = clk.get("sm_mhz") or 0
        print(json.dumps({"probe": name, "iters": iters, "ns_per_group": ns,
                          "cycles_per_group": ns * mhz / 1e3 if mhz else None, "clocks": clk}), flush=True)
    return 0


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--chunks", type=int, default=4096)
    ap.add_argument("--reps", type=int, default=5)
    ap.add_argument("--trace", action="store_true", help="only the timed pair hand-off (per-step SM cycles)")
    ap.add_argument("--latency", action="store_true", help="only the latency probes")
    a = ap.parse_args(argv)
    dev = torch.device("cuda:0")
    if a.trace:
        return trace(dev)
    if a.latency:
        return latency(dev, a.chunks, a.reps)
    probes = [("mma_f16acc", 0, 2), ("mma_f32acc", 1, 2), ("chunk_pipeline_8warp", 2, 2),
              ("chunk_pipeline_16warp", 2, 4), ("pipeline_no_adds_8warp", 3, 2), ("pipeline_no_adds_16warp", 3, 4),
              ("handoff_only_8warp", 4, 2), ("tmem_ld_only_8warp", 6, 2), ("tmem_ld_only_16warp", 6, 4),
              ("tmem_ld_add_8warp", 7, 2), ("tmem_ld_add_16warp", 7, 4),
              ("chunk_pipeline_8warp_spin", 12, 2), ("handoff_only_8warp_spin", 13, 2),
              ("pingpong_no_mma_8warp", 14, 2), ("pingpong_no_mma_8warp_spin", 15, 2),
              ("pingpong_no_mma_8slots", 20, 2), ("mma_f16acc_n64", 21, 2), ("mma_f16acc_n256", 22, 2),
              ("chunk_pipeline_merged_issuer", 23, 2), ("pingpong_no_fence", 24, 2),
              ("pingpong_per_thread_arrive", 25, 2), ("pingpong_no_fence_per_thread", 26, 2),
              ("handoff_per_thread_arrive", 27, 2), ("mma_issue_commit_only", 28, 2),
              ("chunk_pipeline_pairs", 40, 2), ("chunk_pipeline_turn_groups_16warp", 41, 4),
              ("chunk_pipeline_pairs_16warp", 42, 4), ("chunk_pipeline_pairs_16warp_pipelined", 43, 4),
              ("chunk_pipeline_wide_n256_16warp", 45, 4), ("chunk_pipeline_pairs_split_n_16warp", 46, 4)]
    for name, mode, epi in probes:
        sms, ms, tflops, clk = run(mode, epi, a.chunks, a.reps, dev)
        mhz = clk.get("sm_mhz")
        peak = sms * 8192 * mhz * 1e6 / 1e12 if mhz else None
        print(json.dumps({"probe": name, "chunks_per_cta": a.chunks, "ms": ms, "tflops": tflops, "clocks": clk,
                          "frac_of_clock_peak": tflops / peak if peak else None}), flush=True)
    # warp-level mma.sync: 4 blocks of 8 warps per SM, 8 independent chains per warp
    for name, mode in (("mma_sync_f16acc", 30), ("mma_sync_f32acc", 31), ("mma_sync_chunk32", 32),
                       ("mma_sync_smem_64x64_chunked", 33), ("mma_sync_smem_64x64_no_adds", 34),
                       ("mma_sync_smem_64x64_grouped8", 35), ("mma_sync_smem_64x64_grouped16", 36)):
        lib = _lib.load()
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        grid = 4 * sms if mode <= 32 else sms
        out = torch.empty(grid * 256, device=dev)
        iters = max(1024, a.chunks // 4)
        stream = torch.cuda.current_stream(dev)

        def launch():
            rc = lib.f16acc_probe_chunk_rate(mode, 2, iters, grid, out.data_ptr(), dev.index or 0, stream.cuda_stream)
            if rc != 0:
                raise RuntimeError(_lib.strerror(rc))

        launch()
        torch.cuda.synchronize()
        with ClockSampler(dev.index or 0, period_s=0.002) as clocks:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(a.reps):
                launch()
            e1.record(stream)
            torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / a.reps
        mmas_per_warp_iter = {30: 8, 31: 8, 32: 16, 33: 64, 34: 64, 35: 64, 36: 64}[mode]
        tflops = grid * 8 * iters * mmas_per_warp_iter * 4096 / (ms / 1e3) / 1e12
        clk = clocks.summary()
        mhz = clk.get("sm_mhz")
        peak = sms * 8192 * mhz * 1e6 / 1e12 if mhz else None
        print(json.dumps({"probe": name, "iters": iters, "ms": ms, "tflops": tflops, "clocks": clk,
                          "frac_of_clock_peak": tflops / peak if peak else None}), flush=True)
    latency(dev, a.chunks, a.reps)
    st = _lib.load().f16acc_device_status(dev.index or 0, 1)
    if st != 0:
        print(json.dumps({"device_status": st}))
        return 1
    return 0


if __name__ == "__main__":
    sys.exit(main())
