"""The bias epilogue (f16acc_gemm_bias, kernel.mm_bias, patch.linear).

The reference adds the bias after the GEMM (patch.py:28-30: `y = mm(x2,
w.t()); y += b`).  The fused epilogue rounds the product to the output type,
adds the fp16 bias in FP32 and rounds again, which is what the in-place add
does, so every comparison here against `mm` followed by `+= bias` is exact
(torch.equal), in both kernels, both passes (the redo pass rewrites flagged
tiles with the bias too) and every output type and layout.
"""

import numpy as np
import pytest
import torch

import f16acc_b200 as f16acc
from f16acc_b200 import _lib, patch
from f16acc_b200.kernel import mm_bias, mm_ex, plan, tile_flags
from oracle import oracle as O
from tests.test_gpu_parity import VARIANTS, VNAMES, np16, stress, tma_ready

pytestmark = pytest.mark.gpu

OUT_DTYPES = [torch.float16, torch.float32, torch.bfloat16]


def unfused(a, b, bias, out_dtype, chunked, variant, out=None):
    y, _ = mm_ex(a, b, out_dtype, chunked, variant=variant, out=out)
    y += bias
    return y


def operands(M, N, K, seed, device, layout="row_major"):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(M, K, generator=g).half().to(device)
    w = torch.randn(N, K, generator=g).half().to(device)
    b = w.t() if layout == "w_t" else w.t().contiguous()
    bias = (torch.randn(N, generator=g) * 4).half().to(device)
    return a, b, bias


@pytest.mark.parametrize("variant", VARIANTS, ids=VNAMES.get)
@pytest.mark.parametrize("out_dtype", OUT_DTYPES, ids=str)
@pytest.mark.parametrize("chunked", [True, False], ids=["chunked", "fp32acc"])
@pytest.mark.parametrize("layout", ["row_major", "w_t"])
def test_fused_bias_equals_mm_then_add(cuda, variant, out_dtype, chunked, layout):
    a, b, bias = operands(300, 200, 256, seed=11, device=cuda, layout=layout)
    if variant == _lib.VARIANT_TCGEN05:
        a, b = tma_ready(a, b)
    c, _ = mm_ex(a, b, out_dtype, chunked, variant=variant, bias=bias)
    assert torch.equal(c, unfused(a, b, bias, out_dtype, chunked, variant))


@pytest.mark.parametrize("variant", VARIANTS, ids=VNAMES.get)
@pytest.mark.parametrize("M,N", [(129, 77), (1, 8), (260, 136), (128, 1000)])
def test_ragged_n_tails(cuda, variant, M, N):
    a, b, bias = operands(M, N, 96, seed=M + N, device=cuda)
    if variant == _lib.VARIANT_TCGEN05:
        a, b = tma_ready(a, b)
    for dt in OUT_DTYPES:
        c, _ = mm_ex(a, b, dt, variant=variant, bias=bias)
        assert torch.equal(c, unfused(a, b, bias, dt, True, variant))


def test_strided_bias_and_strided_outputs(cuda):
    a, b, _ = operands(200, 160, 128, seed=5, device=cuda)
    bias = (torch.randn(320, device=cuda) * 3).half()[::2]  # element stride 2
    for variant in VARIANTS:
        for dt in (torch.float16, torch.float32):
            ref = unfused(a, b, bias, dt, True, variant)
            wide = torch.full((200, 300), -7.0, device=cuda, dtype=dt)
            out = wide[:, 50:210]
            mm_ex(a, b, dt, variant=variant, out=out, bias=bias)
            assert torch.equal(out, ref)
            assert (wide[:, :50] == -7).all() and (wide[:, 210:] == -7).all()
            colmajor = torch.empty(160, 200, device=cuda, dtype=dt).t()  # element-wise copy-out path
            mm_ex(a, b, dt, variant=variant, out=colmajor, bias=bias)
            assert torch.equal(colmajor, ref)


@pytest.mark.parametrize("variant", VARIANTS, ids=VNAMES.get)
@pytest.mark.parametrize("out_dtype", [torch.float16, torch.float32], ids=str)
def test_redo_pass_adds_the_bias(cuda, variant, out_dtype):
    a, b = stress(512, 640, 384, seed=3)
    a, b = a.to(cuda), b.to(cuda)
    bias = torch.randn(640, device=cuda).half()
    if variant == _lib.VARIANT_TCGEN05:
        a, b = tma_ready(a, b)
    c, ws = mm_ex(a, b, out_dtype, variant=variant, bias=bias)
    flags = tile_flags(ws, plan(a, b, variant)).cpu().numpy()
    assert flags.any() and not flags.all()
    # flags see the product only (the bias cannot raise one), as in the reference
    _, oflags = O.gemm_chunked(np16(a), np16(b), round_every=16, tile=plan(a, b, variant)["tile"], redo=False)
    np.testing.assert_array_equal(flags, oflags.astype(bool))
    assert torch.equal(c, unfused(a, b, bias, out_dtype, True, variant))
    tm, tn = plan(a, b, variant)["tile"]
    c32 = unfused(a, b, bias, out_dtype, False, variant)
    for i, j in zip(*np.nonzero(flags)):
        sl = (slice(i * tm, (i + 1) * tm), slice(j * tn, (j + 1) * tn))
        assert torch.equal(c[sl], c32[sl])


def test_empty_sum_gives_the_bias(cuda):
    a = torch.empty(256, 0, device=cuda).half()
    b = torch.empty(0, 48, device=cuda).half()
    bias = torch.randn(48, device=cuda).half()
    for dt in OUT_DTYPES:
        c = mm_bias(a, b, bias, dt)
        assert torch.equal(c, bias.to(dt).expand(256, 48))


def test_bias_arguments_are_checked(cuda):
    a = torch.randn(128, 64, device=cuda).half()
    b = torch.randn(64, 32, device=cuda).half()
    with pytest.raises(ValueError):
        mm_bias(a, b, torch.randn(31, device=cuda).half())
    with pytest.raises(ValueError):
        mm_bias(a, b, torch.randn(32, device=cuda))  # fp32 bias
    with pytest.raises(ValueError):
        mm_bias(a, b, torch.randn(32).half())  # host bias
    lib = _lib.load()
    c = torch.empty(128, 32, device=cuda).half()
    rc = lib.f16acc_gemm_bias(a.data_ptr(), 64, 1, b.data_ptr(), 32, 1, None, 1, c.data_ptr(), 32, 1,
                              _lib.OUT_F16, 128, 32, 64, 0, None, 0, 0, torch.cuda.current_stream().cuda_stream,
                              _lib.VARIANT_AUTO)
    assert rc == _lib.ERR_INVALID_ARGUMENT


def test_linear_uses_the_fused_bias_with_identical_bits(cuda):
    for k in patch.calls:
        patch.calls[k] = 0
    layer = torch.nn.Linear(384, 640).cuda().half()
    x = torch.randn(2, 150, 384, device=cuda).half()
    f16acc.enable()
    try:
        with torch.no_grad():
            y = layer(x)
    finally:
        f16acc.disable()
    assert patch.calls["chunked"] == 1
    y_ref = f16acc.mm(x.reshape(300, 384), layer.weight.t())
    y_ref += layer.bias  # the reference's patch.py:28-30
    assert torch.equal(y, y_ref.view(2, 150, 640))


def test_linear_keeps_the_unfused_add_for_other_biases(cuda):
    for k in patch.calls:
        patch.calls[k] = 0
    x = torch.randn(256, 64, device=cuda).half()
    w = torch.randn(96, 64, device=cuda).half()
    b32 = torch.randn(96, device=cuda)  # fp32 bias: `y += b` as the reference
    f16acc.enable()
    try:
        with torch.no_grad():
            y = torch.nn.functional.linear(x, w, b32)
    finally:
        f16acc.disable()
    y_ref = f16acc.mm(x, w.t())
    y_ref += b32
    assert patch.calls["chunked"] == 1
    assert torch.equal(y, y_ref)
