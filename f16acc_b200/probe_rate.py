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


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--chunks", type=int, default=4096)
    ap.add_argument("--reps", type=int, default=5)
    a = ap.parse_args(argv)
    dev = torch.device("cuda:0")
    probes = [("mma_f16acc", 0, 2), ("mma_f32acc", 1, 2), ("chunk_pipeline_8warp", 2, 2),
              ("chunk_pipeline_16warp", 2, 4)]
    for name, mode, epi in probes:
        sms, ms, tflops, clk = run(mode, epi, a.chunks, a.reps, dev)
        mhz = clk.get("sm_mhz")
        peak = sms * 8192 * mhz * 1e6 / 1e12 if mhz else None
        print(json.dumps({"probe": name, "chunks_per_cta": a.chunks, "ms": ms, "tflops": tflops, "clocks": clk,
                          "frac_of_clock_peak": tflops / peak if peak else None}), flush=True)
    st = _lib.load().f16acc_device_status(dev.index or 0, 1)
    if st != 0:
        print(json.dumps({"device_status": st}))
        return 1
    return 0


if __name__ == "__main__":
    sys.exit(main())
