"""Host-side behaviour that needs no GPU: the API surface of
steppergg/f16acc (f16acc/__init__.py:8-11, patch.py:17-40) and mm()'s input
checks (kernel.py:85-90)."""

import pytest
import torch

import f16acc_b200 as f16acc
from f16acc_b200 import patch


def test_public_surface_is_the_reference_one():
    assert f16acc.__all__ == ["mm", "enable", "disable", "calls"]
    assert f16acc.calls is patch.calls
    assert patch.MIN_ROWS == 128
    assert patch._orig is torch.nn.functional.linear or patch._orig.__name__ == "linear"


def test_reference_import_name_is_the_same_package():
    # `import f16acc` / `from f16acc import patch` (tests/test_f16acc.py:5-6)
    # give this build's objects, not copies: state is shared both ways
    import importlib

    ref_name = importlib.import_module("f16acc")
    ref_kernel = importlib.import_module("f16acc.kernel")
    from f16acc import patch as ref_patch

    assert ref_name.__all__ == ["mm", "enable", "disable", "calls"]
    assert ref_patch is patch and ref_name.calls is patch.calls
    assert ref_name.mm is f16acc.mm and ref_kernel.mm is f16acc.mm
    ref_name.enable()
    try:
        assert torch.nn.functional.linear is patch.linear
    finally:
        ref_name.disable()
    assert torch.nn.functional.linear is patch._orig


def test_mm_rejects_bad_inputs_with_valueerror():
    a = torch.randn(256, 64).half()
    for bad in (torch.randn(32, 64).half(), torch.randn(64, 64), torch.randn(64, 64).half()):
        with pytest.raises(ValueError):
            f16acc.mm(a, bad)  # shape mismatch, fp32, and CPU tensors
    with pytest.raises(ValueError):
        f16acc.mm(torch.randn(4, 4, 4).half(), torch.randn(4, 4).half())


def test_enable_disable_swap_f_linear():
    f16acc.enable()
    try:
        assert torch.nn.functional.linear is patch.linear
    finally:
        f16acc.disable()
    assert torch.nn.functional.linear is patch._orig


def test_cpu_inputs_fall_back_and_count():
    for k in patch.calls:
        patch.calls[k] = 0
    lin = torch.nn.Linear(16, 8).half()
    f16acc.enable()
    try:
        with torch.no_grad():
            y = lin(torch.randn(300, 16).half())
    finally:
        f16acc.disable()
    assert y.shape == (300, 8)
    assert patch.calls == {"chunked": 0, "original": 1}
