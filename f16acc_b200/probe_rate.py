"""B200 raw-rate probes (counterpart of the reference's bench/rate.py and
bench/chunkrate.py): tcgen05 MMA throughput with an FP16 against an FP32
accumulator, the ceiling of the chunked pipeline (MMA + per-chunk TMEM load +
FP32 add) with no global-memory traffic, and the warp-level mma.sync rates.

    python -m f16acc_b200.probe_rate [--chunks 16384] [--reps 5]

Prints one JSON line per probe: TFLOPS and the fraction of the clock-normalised
dense peak 148 SMs x 8192 flop/clk x the SM clock NVML reports during the run.
"""

from __future__ import annotations

import argparse
import json
import statistics
import sys

import torch

from . import _lib
from .nvml import ClockSampler

# mode -> (name, epi_split, flops per CTA (tcgen05) or per warp (mma.sync) per iteration)
PROBES = [
    (0, "tcgen05 MMA only, FP16 accumulator", 2, 2.0 * 128 * 128 * 32),
    (1, "tcgen05 MMA only, FP32 accumulator", 2, 2.0 * 128 * 128 * 32),
    (2, "chunk-pair pipeline, 8 epilogue warps (MMA + TMEM load + FP32 add)", 2, 2.0 * 128 * 128 * 32),
    (2, "chunk-pair pipeline, 16 epilogue warps", 4, 2.0 * 128 * 128 * 32),
    (30, "mma.sync m16n8k16, FP16 accumulate (8 chains per warp)", 0, 8 * 4096.0),
    (31, "mma.sync m16n8k16, FP32 accumulate (8 chains per warp)", 0, 8 * 4096.0),
    (32, "mma.sync, FP16 chunks of 2 K16 steps added into FP32 (chunkrate analogue)", 0, 8 * 8192.0),
]


def run(mode: int, epi_split: int, chunks: int, reps: int, dev: torch.device, flops_unit: float):
    lib = _lib.load()
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    warp_level = mode >= 30
    grid = sms * 4 if warp_level else sms  # mma.sync: 4 blocks of 8 warps per SM
    threads = 256 if warp_level else 96 + 128 * epi_split
    out = torch.empty(grid * threads, device=dev)
    stream = torch.cuda.current_stream(dev)

    def launch():
        rc = lib.f16acc_probe_chunk_rate(mode, max(epi_split, 2), chunks, grid, out.data_ptr(), dev.index or 0,
                                         stream.cuda_stream)
        if rc != _lib.OK:
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
    units = grid * 8 if warp_level else grid  # warps or CTAs
    flops = units * chunks * flops_unit
    return sms, med, flops / (med / 1e3) / 1e12, clocks.summary()


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--chunks", type=int, default=16384)
    ap.add_argument("--reps", type=int, default=5)
    a = ap.parse_args(argv)
    dev = torch.device("cuda:0")
    for mode, name, epi, unit in PROBES:
        sms, ms, tflops, clk = run(mode, epi, a.chunks, a.reps, dev, unit)
        mhz = clk.get("sm_mhz") or clk.get("sm_max_mhz") or 1965.0
        peak = sms * 8192 * mhz * 1e6 / 1e12
        print(json.dumps({"mode": mode, "probe": name, "epi_split": epi or None, "chunks": a.chunks, "ms": ms,
                          "tflops": tflops, "peak_tflops_at_clock": peak, "frac": tflops / peak, "clocks": clk}),
              flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
