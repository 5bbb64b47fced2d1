"""BASELINE configs 2, 3 and 5 at their full sizes, checked element by element
against the CPU oracle on sampled rows (the oracle finishes a few hundred
rows of these products in seconds) and against an FP64 product.

Tolerances (as in test_gpu_parity.py): a chunked result may differ from the
oracle's round-after-each-K16 emulation by 2 FP16 ulps of every chunk's
absolute sum plus FP32 rounding of the running sum; an fp16 output adds at
most one FP16 rounding of the value (two where an fp16 bias is added after
the product is rounded, as the reference's `y += b` does).
"""

import numpy as np
import pytest
import torch

import f16acc_b200 as f16acc
from f16acc_b200 import _lib, patch
from f16acc_b200.kernel import plan
from oracle import oracle as O
from tests.helpers import chunk_ulp_bound_torch, ulp16

pytestmark = pytest.mark.gpu


def sample_rows(m, count, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.sort(torch.randperm(m, generator=g)[:count]).values


def check_rows_against_oracle(c, a, b, rows, extra_ulps=1.0):
    """c[rows] against the oracle's chunked product of a[rows] @ b."""
    a_s = a[rows]
    ref, _ = O.gemm_chunked(a_s.cpu().numpy(), b.cpu().numpy(), round_every=16)
    bound = chunk_ulp_bound_torch(a_s, b).cpu().numpy()
    ref = ref.astype(np.float64)
    if c.dtype == torch.float16:
        bound = bound + extra_ulps * ulp16(ref)
    got = c[rows].double().cpu().numpy()
    err = np.abs(got - ref)
    assert np.isfinite(got).all()
    worst = np.unravel_index(np.argmax(err - bound), err.shape)
    assert (err <= bound).all(), f"err {err[worst]} > bound {bound[worst]} at {worst}"


def fp64_rel(c, a, b):
    ref = a.double() @ b.double()
    return ((c.double() - ref).abs().max() / ref.abs().max()).item()


@pytest.mark.parametrize("layout", ["row_major", "w_t"])
@pytest.mark.parametrize("out_dtype", [torch.float16, torch.float32], ids=str)
def test_config2_4096_rows_match_the_oracle(cuda, layout, out_dtype):
    # 4096^3, N(0,1)/sqrt(K)*4 seed 1, B row-major or w.t()
    n = 4096
    g = torch.Generator(device=cuda).manual_seed(1)
    a = (torch.randn(n, n, device=cuda, generator=g) / n ** 0.5 * 4).half()
    b = (torch.randn(n, n, device=cuda, generator=g) / n ** 0.5 * 4).half()
    if layout == "w_t":
        b = b.t().contiguous().t()
    assert plan(a, b)["variant"] == _lib.VARIANT_TCGEN05
    c = f16acc.mm(a, b, out_dtype)
    assert fp64_rel(c, a, b) <= 1e-3
    check_rows_against_oracle(c, a, b, sample_rows(n, 256, seed=2))


QWEN_SHAPES = [("q_o_proj", 1536, 1536), ("k_v_proj", 1536, 256), ("gate_up_proj", 1536, 8960),
               ("down_proj", 8960, 1536), ("lm_head", 1536, 151936)]


@pytest.mark.parametrize("name,K,N", QWEN_SHAPES, ids=[s[0] for s in QWEN_SHAPES])
def test_config3_qwen_shapes(cuda, name, K, N):
    # M = 2048, x ~ N(0,1), W [N, K] ~ N(0, 0.02), seed 2, y = mm(x, W.t())
    M = 2048
    g = torch.Generator(device=cuda).manual_seed(2)
    x = torch.randn(M, K, device=cuda, generator=g).half()
    w = (torch.randn(N, K, device=cuda, generator=g) * 0.02).half()
    y = f16acc.mm(x, w.t())
    assert y.dtype == torch.float16 and y.shape == (M, N)
    assert fp64_rel(y, x, w.t()) <= 1e-3
    check_rows_against_oracle(y, x, w.t(), sample_rows(M, 64 if N > 100000 else 256, seed=3))


def test_config5_routed_qwen2_two_layers(cuda):
    """BASELINE config 5 at the real widths with 2 of the 28 decoder layers:
    random-init Qwen2.5-1.5B architecture (N(0, 0.02) fp16 weights, seed 4), one
    2048-token prompt of uniform-random ids, every nn.Linear routed through
    f16acc.enable().  Each routed call's output matches the oracle on sampled
    rows, every linear is routed, and the top-1 predictions agree with the
    cuBLAS FP32-accumulate run."""
    transformers = pytest.importorskip("transformers")
    from f16acc_b200.workloads import qwen2_config

    cfg = qwen2_config()
    cfg.num_hidden_layers = 2
    torch.manual_seed(4)
    with torch.device(cuda):
        model = transformers.Qwen2ForCausalLM(cfg).half().eval()
    g = torch.Generator(device=cuda).manual_seed(5)
    ids = torch.randint(0, cfg.vocab_size, (1, 2048), device=cuda, generator=g)
    rows = sample_rows(2048, 16, seed=6)
    seen = []

    def hook(mod, inp, out):
        x = inp[0].reshape(-1, inp[0].shape[-1])
        y = out.reshape(-1, out.shape[-1])
        bias = mod.bias.detach().double().cpu().numpy() if mod.bias is not None else None
        seen.append((x[rows].cpu(), mod.weight.detach(), bias, y[rows].cpu()))

    linears = [m for m in model.modules() if isinstance(m, torch.nn.Linear)]
    torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = False
    with torch.no_grad():
        patch.disable()
        top1_cublas = model(ids).logits[0].argmax(-1)
        for k in patch.calls:
            patch.calls[k] = 0
        handles = [m.register_forward_hook(hook) for m in linears]
        f16acc.enable()
        try:
            top1_f16acc = model(ids).logits[0].argmax(-1)
        finally:
            f16acc.disable()
            for h in handles:
                h.remove()
    # 7 linears per layer (q, k, v, o, gate, up, down) and the tied lm_head, all routed
    assert len(seen) == 2 * 7 + 1
    assert patch.calls == {"chunked": 15, "original": 0}
    for x_s, w, bias, y_s in seen:
        b = w.t()
        ref, _ = O.gemm_chunked(x_s.numpy(), b.cpu().numpy(), round_every=16)
        ref = ref.astype(np.float64)
        bound = chunk_ulp_bound_torch(x_s.to(cuda), b).cpu().numpy() + ulp16(ref)
        if bias is not None:
            ref = ref + bias
            bound = bound + ulp16(ref)
        err = np.abs(y_s.double().numpy() - ref)
        assert (err <= bound).all(), (tuple(w.shape), float(err.max()))
    agree = (top1_f16acc == top1_cublas).float().mean().item()
    print(f"\ntop-1 agreement with cuBLAS FP32 accumulate: {agree:.4f}")
    assert agree >= 0.95
