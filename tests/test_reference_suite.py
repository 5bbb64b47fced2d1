"""The reference's own test suite (steppergg/f16acc tests/test_f16acc.py),
re-run against this build: same inputs, same thresholds, same API calls, and
the reference's own imports (`import f16acc`, `from f16acc import patch`,
tests/test_f16acc.py:5-6), which resolve to this build's drop-in package."""

import pytest
import torch

import f16acc
from f16acc import patch

pytestmark = pytest.mark.gpu


def rel(x, ref):
    return ((x.double() - ref).abs().max() / ref.abs().max()).item()


# ---------------------------------------------------------------- class Kernel (:15-62)

def test_odd_sizes_match_fp64(cuda):  # :21-24
    a = torch.randn(1000, 777, device="cuda").half()
    b = torch.randn(777, 1234, device="cuda").half()
    assert rel(f16acc.mm(a, b, torch.float32), a.double() @ b.double()) < 2e-3


def test_close_to_fp32_accumulate_and_better_than_plain_fp16(cuda):  # :26-40
    torch.manual_seed(0)
    a = torch.randn(4096, 4096, device="cuda").half()
    b = torch.randn(4096, 4096, device="cuda").half()
    ref = a.double() @ b.double()
    m = torch.backends.cuda.matmul
    fp32 = rel(torch.mm(a, b), ref)
    m.allow_fp16_accumulation = True
    try:
        plain = rel(torch.mm(a, b), ref)
    finally:
        m.allow_fp16_accumulation = False
    ours = rel(f16acc.mm(a, b), ref)
    assert ours < 3 * fp32  # reference measured 4.8e-4 vs 3.6e-4 on Ada
    assert ours * 5 < plain  # reference measured 4.8e-4 vs 8.8e-3 on Ada


def test_bad_inputs_raise_instead_of_reading_out_of_bounds(cuda):  # :42-47
    a = torch.randn(256, 64, device="cuda").half()
    for bad in (torch.randn(32, 64, device="cuda").half(), torch.randn(64, 64, device="cuda"),
                torch.randn(64, 64).half()):
        with pytest.raises(ValueError):
            f16acc.mm(a, bad)


@pytest.mark.slow
def test_output_past_2_31_elements_is_addressed_correctly(cuda):  # :49-57
    if torch.cuda.mem_get_info()[0] <= 6 * 2 ** 30:
        pytest.skip("needs about 5 GB free VRAM")
    x = torch.randn(14200, 1536, device="cuda").half() * 0.1
    w = torch.randn(151936, 1536, device="cuda").half() * 0.1
    c = f16acc.mm(x, w.t())
    assert rel(c[-4:], (x[-4:] @ w.t()).double()) < 1e-2
    del c, x, w
    torch.cuda.empty_cache()


def test_transposed_weight_view(cuda):  # :59-62
    x = torch.randn(256, 384, device="cuda").half()
    w = torch.randn(640, 384, device="cuda").half()
    assert rel(f16acc.mm(x, w.t()), x.double() @ w.double().t()) < 2e-3


# ---------------------------------------------------------------- class Patch (:65-116)

@pytest.fixture
def lin(cuda):
    for k in patch.calls:
        patch.calls[k] = 0
    layer = torch.nn.Linear(384, 640).cuda().half()
    f16acc.enable()
    yield layer
    f16acc.disable()


def test_linear_routed_with_bias_and_batch_dims(lin):  # :76-83
    x = torch.randn(2, 150, 384, device="cuda").half()
    with torch.no_grad():
        y = lin(x)
    ref = x.double() @ lin.weight.double().t() + lin.bias.double()
    assert y.shape == (2, 150, 640)
    assert rel(y, ref) < 2e-3
    assert patch.calls["chunked"] == 1


def test_small_and_grad_inputs_fall_back(lin):  # :85-89
    with torch.no_grad():
        lin(torch.randn(8, 384, device="cuda").half())
    lin(torch.randn(256, 384, device="cuda").half())  # grad enabled
    assert patch.calls == {"chunked": 0, "original": 2}


def test_fp16_chunk_overflow_is_redone_with_fp32_accumulate(lin):  # :91-101
    layer = torch.nn.Linear(64, 128, bias=False).cuda().half()
    with torch.no_grad():
        layer.weight[:, :32] = 30.0
        layer.weight[:, 32:] = -30.0
        layer.weight[:, 63] = -29.0
        y = layer(torch.full((256, 64), 100.0, device="cuda").half())
    assert patch.calls["chunked"] == 1
    assert torch.all(y == 100.0)


def test_no_overflow_leaves_flags_clear(lin):  # :103-106
    x = torch.randn(300, 384, device="cuda").half()
    w = torch.randn(384, 500, device="cuda").half()
    assert torch.isfinite(f16acc.mm(x, w)).all()


def test_zero_width_layer_does_not_crash(lin):  # :108-112, plus the value the reference leaves unchecked
    layer = torch.nn.Linear(0, 16).cuda().half()
    with torch.no_grad():
        y = layer(torch.empty(256, 0, device="cuda").half())
    assert y.shape == (256, 16)
    assert torch.equal(y, layer.bias.expand(256, 16))  # empty sum is 0, plus the bias


def test_disable_restores_original(lin):  # :114-116
    f16acc.disable()
    assert torch.nn.functional.linear is patch._orig
