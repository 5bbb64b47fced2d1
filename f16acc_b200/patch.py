"""Linear-layer routing: `enable()` makes every qualifying torch linear call
run on the chunked GEMM of this package; `disable()` puts cuBLAS back.

The hook point is `torch.nn.functional.linear`, the function nn.Linear's
forward looks up at call time, so patching that one attribute covers every
nn.Linear in every model.  The routing rule is the reference's
(steppergg/f16acc f16acc/patch.py:22-32, kept unchanged for drop-in
behaviour): a call is routed only when the input is fp16 on a CUDA device,
the weight is fp16, no autograd graph is being recorded, and the flattened
input has at least MIN_ROWS rows; anything else (CPU tensors, other dtypes,
training, few-row decode steps) goes to the saved original.  Overflowing
tiles are repaired on the device, so a routed call never synchronises with
the host.  One change from the reference: an fp16 bias of shape
(out_features,) is applied by the GEMM's epilogue instead of by a second
in-place pass over the output; the bits are the same.
"""

import torch
import torch.nn.functional as F

from .kernel import mm, mm_bias

MIN_ROWS = 128
_orig = F.linear
calls = {"chunked": 0, "original": 0}


def linear(x, w, b=None):
    rows = x.shape[:-1].numel()
    if not (x.is_cuda and x.dtype == w.dtype == torch.float16 and rows >= MIN_ROWS and not torch.is_grad_enabled()):
        calls["original"] += 1
        return _orig(x, w, b)
    x2 = x.reshape(rows, x.shape[-1])
    n = w.shape[0]
    if b is not None and b.dtype == torch.float16 and b.device == x.device and b.shape == (n,):
        # Bias added in the GEMM epilogue; bit-identical to `y += b` after mm.
        y = mm_bias(x2, w.t(), b)
    else:
        y = mm(x2, w.t())  # [K, N] view of the [N, K] weight: K-contiguous B, no copy
        if b is not None:
            y += b
    calls["chunked"] += 1
    return y.view(*x.shape[:-1], w.shape[0])


def enable():
    F.linear = linear  # the attribute nn.Linear.forward resolves on every call


def disable():
    F.linear = _orig
