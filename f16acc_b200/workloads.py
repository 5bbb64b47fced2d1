"""The BASELINE workloads beyond the headline GEMM, run by `bench.py --workload`.

    shapes    config 3: Qwen2.5-1.5B linear shapes at M=2048, weight [N, K]
              (nn.Linear layout), per-shape TFLOPS vs cuBLAS FP32 accumulate
              (the reference's bench/shapes.py measurement)
    overflow  config 4: 4096^3 N(0,1) with 1% of A rows and B columns x64 --
              flagged-tile fraction and redo cost; plus 4b, a controlled case
              with about 1% of tiles flagged, overhead against the same shape
              with no scaling
    nshard    config 4c: N-column-sharded 16384^3 over the ranks of a torchrun
              job, NCCL all-gather of C (`shard.nshard_mm`)
    prefill   config 5: random-init Qwen2.5-1.5B architecture, 2048-token
              prompts, every nn.Linear through `f16acc.enable()`; tokens/s and
              top-1 agreement against the cuBLAS FP32-accumulate run

Timing: CUDA events on the current stream.  Where one product's operands fit
in L2, each timed repetition is preceded by an L2 flush (a 256 MiB write)
outside its event pair, and the median is reported.
"""

from __future__ import annotations

import statistics

import torch

from . import _lib
from .kernel import mm, mm_ex, plan, tile_flags

L2_FLUSH_BYTES = 256 << 20


class L2Flusher:
    def __init__(self, device):
        self.buf = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=device)

    def __call__(self):
        self.buf.fill_(1.0)


def time_op(op, reps: int, flush: L2Flusher | None, warmup: int = 3) -> float:
    """Median milliseconds of op() over `reps` event-timed calls."""
    for _ in range(warmup):
        op()
    torch.cuda.synchronize()
    ms = []
    for _ in range(reps):
        if flush is not None:
            flush()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        op()
        e1.record()
        ms.append((e0, e1))
    torch.cuda.synchronize()
    return statistics.median(a.elapsed_time(b) for a, b in ms)


def rel(x, ref) -> float:
    return ((x.double() - ref).abs().max() / ref.abs().max()).item()


# ---------------------------------------------------------------- config 3
QWEN_SHAPES = [("q_o_proj", 1536, 1536), ("k_v_proj", 1536, 256), ("gate_up_proj", 1536, 8960),
               ("down_proj", 8960, 1536), ("lm_head", 1536, 151936)]


def shapes(device, reps: int = 20, M: int = 2048, seed: int = 2):
    torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = False
    flush = L2Flusher(device)
    g = torch.Generator(device=device).manual_seed(seed)
    out = []
    for name, K, N in QWEN_SHAPES:
        x = torch.randn(M, K, device=device, generator=g).half()
        w = (torch.randn(N, K, device=device, generator=g) * 0.02).half()
        flops = 2.0 * M * N * K
        t_cublas = time_op(lambda: torch.nn.functional.linear(x, w), reps, flush)
        t_ours = time_op(lambda: mm(x, w.t()), reps, flush)
        c = mm(x, w.t())
        err = rel(c, x.double() @ w.double().t())
        bytes_alg = 2 * (M * K + N * K + M * N)
        out.append({"shape": name, "M": M, "K": K, "N": N, "ours_tflops": flops / t_ours / 1e9,
                    "cublas_f32acc_tflops": flops / t_cublas / 1e9, "speedup_vs_cublas": t_cublas / t_ours,
                    "ours_ms": t_ours, "ours_gbs": bytes_alg / t_ours / 1e6, "max_rel_err_vs_fp64": err,
                    "kernel": _lib.VARIANT_NAMES[plan(x, w.t())["variant"]]})
    return out


# ---------------------------------------------------------------- few rows (decode shapes)
def graph_time(fns) -> float:
    """Per-call device milliseconds of the calls in `fns` replayed from one CUDA
    graph (no host launch overhead in the number)."""
    for f in fns:
        f()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for f in fns:
            f()
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(3):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / (3 * len(fns))


def decode(device, rows=(1, 16, 32, 64), hbm_gbs: float | None = None, calls: int = 24, seed: int = 5):
    """Few-row products (M = batch of decode tokens) on the Qwen2.5-1.5B weight
    shapes: the few-row kernel against the tcgen05 kernel and cuBLAS, in GB/s
    of algorithmic bytes (A + B + C) and as a fraction of the HBM peak.  Each
    timing replays `calls` products over weight copies that together exceed L2."""
    torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = False
    g = torch.Generator(device=device).manual_seed(seed)
    out = []
    for M in rows:
        for name, K, N in QWEN_SHAPES:
            copies = max(1, min(calls, (300 << 20) // (2 * K * N) + 1))
            ws = [(torch.randn(N, K, device=device, generator=g) * 0.02).half() for _ in range(copies)]
            x = torch.randn(M, K, device=device, generator=g).half()
            byts = 2 * (M * K + K * N + M * N)
            res = {"shape": name, "M": M, "K": K, "N": N, "kernel": _lib.VARIANT_NAMES[plan(x, ws[0].t())["variant"]]}
            arms = (("f16acc", lambda w: (lambda: mm(x, w.t()))),
                    ("f16acc_tcgen05", lambda w: (lambda: mm_ex(x, w.t(), variant=_lib.VARIANT_TCGEN05))),
                    ("cublas", lambda w: (lambda: torch.nn.functional.linear(x, w))))
            for arm, make in arms:
                ms = graph_time([make(ws[i % copies]) for i in range(calls)])
                res[arm + "_us"] = ms * 1e3
                res[arm + "_gbs"] = byts / (ms / 1e3) / 1e9
                if hbm_gbs:
                    res[arm + "_frac_hbm"] = res[arm + "_gbs"] / hbm_gbs
            c = mm(x, ws[0].t())
            res["max_rel_err_vs_fp64"] = rel(c, x.double() @ ws[0].double().t())
            out.append(res)
            del ws
    return out


# ---------------------------------------------------------------- config 4 / 4b
def _stress_inputs(device, n, seed, rows, cols, scale=64.0):
    g = torch.Generator(device=device).manual_seed(seed)
    a = torch.randn(n, n, device=device, generator=g)
    b = torch.randn(n, n, device=device, generator=g)
    a[rows] *= scale
    b[:, cols] *= scale
    return a.half(), b.half()


def overflow(device, reps: int = 20, n: int = 4096, seed: int = 3):
    flush = L2Flusher(device)
    g = torch.Generator().manual_seed(seed)
    k = max(1, n // 100)
    out = {}
    lib = _lib.load()
    modes = {"inline": _lib.REDO_INLINE, "separate": _lib.REDO_SEPARATE}

    def timed_modes(a, b):
        """ms of mm(a, b) per redo mode; the library's mode is restored after."""
        res = {}
        for name, mode in modes.items():
            prev = lib.f16acc_set_redo_mode(mode)
            try:
                res[name] = time_op(lambda: mm(a, b), reps, flush)
            finally:
                lib.f16acc_set_redo_mode(prev)
        return res

    base_a, base_b = _stress_inputs(device, n, seed, [], [], 1.0)
    t_base = timed_modes(base_a, base_b)
    cases = {
        # 1% of rows and of columns, chosen by seed, x64
        "config4_random_1pct_rows_cols": (torch.randperm(n, generator=g)[:k].tolist(),
                                          torch.randperm(n, generator=g)[:k].tolist()),
        # 4b: the scaled rows inside one 128-row tile band and the scaled columns inside
        # one 1024-column band, so about 1% of the tiles overflow
        "config4b_controlled_1pct_tiles": (list(range(0, 32)), list(range(0, 1024, 8))),
    }
    for name, (rows, cols) in cases.items():
        a, b = _stress_inputs(device, n, seed, rows, cols)
        c, ws = mm_ex(a, b, torch.float16)
        c32, _ = mm_ex(a, b, torch.float16, chunked=False)
        pl = plan(a, b)
        flags = tile_flags(ws, pl)
        tm, tn = pl["tile"]
        mask = flags.repeat_interleave(tm, 0).repeat_interleave(tn, 1)[:n, :n]
        redone_equal = bool(torch.equal(c[mask], c32[mask]))
        t = timed_modes(a, b)
        # the default (in-kernel) redo is the headline; the reference-shaped second launch beside it
        out[name] = {"flagged_tiles": int(flags.sum()), "tiles": int(flags.numel()),
                     "flagged_fraction": float(flags.float().mean()), "ms": t["inline"],
                     "ms_no_overflow_same_shape": t_base["inline"], "redo_overhead": t["inline"] / t_base["inline"] - 1.0,
                     "redone_tiles_equal_fp32_path": redone_equal, "tflops": 2.0 * n ** 3 / t["inline"] / 1e9,
                     "separate_redo_launch": {"ms": t["separate"], "ms_no_overflow_same_shape": t_base["separate"],
                                              "redo_overhead": t["separate"] / t_base["separate"] - 1.0}}
    return out


# ---------------------------------------------------------------- config 5
def qwen2_config():
    from transformers import Qwen2Config

    return Qwen2Config(vocab_size=151936, hidden_size=1536, intermediate_size=8960, num_hidden_layers=28,
                       num_attention_heads=12, num_key_value_heads=2, max_position_embeddings=32768,
                       rope_theta=1000000.0, rms_norm_eps=1e-6, tie_word_embeddings=True,
                       initializer_range=0.02, torch_dtype="float16")


def prefill(device, prompts: int = 8, seq: int = 2048, seed: int = 4, rank: int = 0, world: int = 1, reps: int = 3):
    """Random-init Qwen2.5-1.5B architecture; `prompts` prompts split over the
    ranks (data parallel); tokens/s for cuBLAS (FP32 accumulate) and for
    every nn.Linear routed through f16acc, plus top-1 agreement."""
    from transformers import Qwen2ForCausalLM

    from . import patch

    torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = False
    torch.manual_seed(seed)
    with torch.device(device):
        model = Qwen2ForCausalLM(qwen2_config()).half().eval()
    mine = [p for p in range(prompts) if p % world == rank]
    g = torch.Generator(device=device).manual_seed(seed + 1)
    ids = torch.randint(0, 151936, (prompts, seq), device=device, generator=g)[mine]

    def run_all():
        outs = []
        with torch.no_grad():
            for i in range(ids.shape[0]):
                outs.append(model(ids[i:i + 1]).logits[0].argmax(-1))
        return outs

    res = {}
    for name, on in (("cublas_f32acc", False), ("f16acc", True)):
        patch.enable() if on else patch.disable()
        for k in patch.calls:
            patch.calls[k] = 0
        top1 = run_all()  # warm-up, and the predictions
        torch.cuda.synchronize()
        times = []
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            run_all()
            e1.record()
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1))
        res[name] = {"ms": statistics.median(times), "top1": top1, "calls": dict(patch.calls)}
    patch.disable()
    agree = torch.cat([(a == b).float() for a, b in zip(res["f16acc"]["top1"], res["cublas_f32acc"]["top1"])])
    tokens = len(mine) * seq
    return {"prompts_on_rank": len(mine), "tokens_on_rank": tokens,
            "ms_cublas": res["cublas_f32acc"]["ms"], "ms_f16acc": res["f16acc"]["ms"],
            "top1_agreement": float(agree.mean()), "routed_calls_per_pass": res["f16acc"]["calls"]}
