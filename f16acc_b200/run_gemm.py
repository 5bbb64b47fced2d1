"""Run one chunked GEMM shape a few times and report time, TFLOPS and error.

    python -m f16acc_b200.run_gemm --m 4096 --n 4096 --k 4096 [--layout row_major|w_t]
        [--variant auto|tcgen05|mma_sync] [--fp32-acc] [--out f16|f32] [--reps 10]

A small command-line check of one shape on cuda:0 (also the command profiles
are taken with: it launches little besides the GEMM itself).
"""

from __future__ import annotations

import argparse
import json
import statistics
import sys

import torch

from . import _lib
from .kernel import mm_ex, plan


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--m", type=int, default=4096)
    ap.add_argument("--n", type=int, default=4096)
    ap.add_argument("--k", type=int, default=4096)
    ap.add_argument("--layout", choices=["row_major", "w_t"], default="row_major")
    ap.add_argument("--variant", choices=["auto", "tcgen05", "mma_sync", "skinny"], default="auto")
    ap.add_argument("--fp32-acc", action="store_true", help="chunked=False (plain FP32 accumulation)")
    ap.add_argument("--out", choices=["f16", "f32"], default="f16")
    ap.add_argument("--reps", type=int, default=10)
    ap.add_argument("--seed", type=int, default=1)
    ap.add_argument("--check", action="store_true", help="max rel err vs an FP64 product")
    ap.add_argument("--epi", type=int, default=None, help="tcgen05 epilogue column slices per lane quarter (2 or 4)")
    a = ap.parse_args(argv)
    if a.epi is not None and _lib.load().f16acc_set_tc_config(128, a.epi) != 0:
        raise SystemExit(f"unsupported --epi {a.epi}")

    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev).manual_seed(a.seed)
    scale = 4.0 / a.k ** 0.5
    A = (torch.randn(a.m, a.k, device=dev, generator=g) * scale).half()
    if a.layout == "row_major":
        B = (torch.randn(a.k, a.n, device=dev, generator=g) * scale).half()
    else:
        B = (torch.randn(a.n, a.k, device=dev, generator=g) * scale).half().t()
    variant = {v: k for k, v in _lib.VARIANT_NAMES.items()}[a.variant]
    out_dtype = torch.float16 if a.out == "f16" else torch.float32
    chunked = not a.fp32_acc
    C, ws = mm_ex(A, B, out_dtype, chunked, variant=variant)
    torch.cuda.synchronize()
    times = []
    for _ in range(a.reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        mm_ex(A, B, out_dtype, chunked, variant=variant, out=C, workspace=ws)
        e1.record()
        times.append((e0, e1))
    torch.cuda.synchronize()
    ms = [e0.elapsed_time(e1) for e0, e1 in times]
    med = statistics.median(ms)
    res = {"m": a.m, "n": a.n, "k": a.k, "layout": a.layout, "chunked": chunked, "out": a.out,
           "variant": _lib.VARIANT_NAMES[plan(A, B, variant)["variant"]],
           "median_ms": med, "tflops": 2.0 * a.m * a.n * a.k / (med / 1e3) / 1e12}
    if a.check:
        ref = A.double() @ B.double()
        res["max_rel_err"] = ((C.double() - ref).abs().max() / ref.abs().max()).item()
    print(json.dumps(res))
    return 0


if __name__ == "__main__":
    sys.exit(main())
