"""The in-kernel redo of flagged tiles (F16ACC_REDO_INLINE, the default).

The reference redoes flagged tiles in a second launch (kernel.py:100-104).
Here each CTA of the chunked tcgen05 kernel recomputes its own flagged tiles in
FP32 mode after its main tiles.  It must give exactly the bits of the
two-launch form (F16ACC_REDO_SEPARATE, and f16acc_gemm_main followed by
f16acc_gemm_redo), whose redone tiles in turn equal the chunked=False output.
"""

import contextlib

import numpy as np
import pytest
import torch

from f16acc_b200 import _lib
from f16acc_b200.kernel import mm_ex, mm_phase, plan, tile_flags
from tests.test_gpu_parity import stress, tma_ready

pytestmark = pytest.mark.gpu


@contextlib.contextmanager
def redo_mode(mode):
    lib = _lib.load()
    prev = lib.f16acc_set_redo_mode(mode)
    assert prev in (_lib.REDO_SEPARATE, _lib.REDO_INLINE)
    try:
        yield
    finally:
        lib.f16acc_set_redo_mode(prev)


@contextlib.contextmanager
def sm_limit(n):
    lib = _lib.load()
    prev = lib.f16acc_set_sm_limit(n)
    try:
        yield
    finally:
        lib.f16acc_set_sm_limit(prev)


def both_modes(a, b, out_dtype, **kw):
    with redo_mode(_lib.REDO_INLINE):
        c1, ws1 = mm_ex(a, b, out_dtype, variant=_lib.VARIANT_TCGEN05, **kw)
    with redo_mode(_lib.REDO_SEPARATE):
        c2, ws2 = mm_ex(a, b, out_dtype, variant=_lib.VARIANT_TCGEN05, **kw)
    return c1, ws1, c2, ws2


def check_redone(c, ws, a, b, out_dtype, **kw):
    pl = plan(a, b, _lib.VARIANT_TCGEN05)
    flags = tile_flags(ws, pl).cpu().numpy()
    c32, _ = mm_ex(a, b, out_dtype, chunked=False, variant=_lib.VARIANT_TCGEN05, **kw)
    tm, tn = pl["tile"]
    for i, j in zip(*np.nonzero(flags)):
        sl = (slice(i * tm, (i + 1) * tm), slice(j * tn, (j + 1) * tn))
        assert torch.equal(c[sl], c32[sl]), f"tile {(i, j)}"
    return flags


@pytest.mark.parametrize("out_dtype", [torch.float16, torch.float32, torch.bfloat16], ids=str)
@pytest.mark.parametrize("layout", ["row_major", "w_t"])
def test_inline_equals_separate_bitwise(cuda, out_dtype, layout):
    a, b = stress(640, 768, 512, seed=21)
    a, b = a.to(cuda), b.to(cuda)
    if layout == "w_t":
        b = b.t().contiguous().t()
    a, b = tma_ready(a, b)
    c1, ws1, c2, ws2 = both_modes(a, b, out_dtype)
    assert torch.equal(c1, c2)
    pl = plan(a, b, _lib.VARIANT_TCGEN05)
    f1, f2 = tile_flags(ws1, pl), tile_flags(ws2, pl)
    assert torch.equal(f1, f2) and f1.any() and not f1.all()
    check_redone(c1, ws1, a, b, out_dtype)


def test_split_main_redo_api_equals_one_call(cuda):
    a, b = stress(512, 512, 384, seed=22)
    a, b = tma_ready(a.to(cuda), b.to(cuda))
    c, _ = mm_ex(a, b, torch.float16, variant=_lib.VARIANT_TCGEN05)
    out = torch.empty_like(c)
    ws = torch.empty(int(_lib.load().f16acc_workspace_bytes(512, 512, 384)), dtype=torch.uint8, device=cuda)
    mm_phase("main", a, b, out, ws, variant=_lib.VARIANT_TCGEN05)
    after_main = out.clone()
    mm_phase("redo", a, b, out, ws, variant=_lib.VARIANT_TCGEN05)
    assert torch.equal(out, c)
    assert not torch.equal(after_main, c)  # the main launch alone leaves flagged tiles to the redo


def test_inline_with_bias_and_strided_output(cuda):
    a, b = stress(384, 520, 256, seed=23)
    a, b = tma_ready(a.to(cuda), b.to(cuda))
    bias = torch.randn(520, device=cuda).half()
    colmajor1 = torch.empty(520, 384, device=cuda).t()
    colmajor2 = torch.empty(520, 384, device=cuda).t()
    with redo_mode(_lib.REDO_INLINE):
        _, ws = mm_ex(a, b, torch.float32, variant=_lib.VARIANT_TCGEN05, out=colmajor1, bias=bias)
    with redo_mode(_lib.REDO_SEPARATE):
        mm_ex(a, b, torch.float32, variant=_lib.VARIANT_TCGEN05, out=colmajor2, bias=bias)
    assert torch.equal(colmajor1, colmajor2)
    assert tile_flags(ws, plan(a, b, _lib.VARIANT_TCGEN05)).any()
    check_redone(colmajor1, ws, a, b, torch.float32, bias=bias)


@contextlib.contextmanager
def schedule(mode):
    lib = _lib.load()
    prev = lib.f16acc_set_schedule(mode)
    assert prev in (_lib.SCHEDULE_STATIC, _lib.SCHEDULE_DYNAMIC)
    try:
        yield
    finally:
        lib.f16acc_set_schedule(prev)


def run_all_orders(a, b, out_dtype):
    """The product under every (tile order, redo mode) pair; first = the defaults."""
    outs = []
    for order in (_lib.SCHEDULE_DYNAMIC, _lib.SCHEDULE_STATIC):
        with schedule(order):
            c1, ws1, c2, _ = both_modes(a, b, out_dtype)
        outs += [(c1, ws1), (c2, None)]
    return outs


@pytest.mark.parametrize("out_dtype", [torch.float16, torch.float32], ids=str)
def test_tile_orders_and_redo_modes_agree_bitwise(cuda, out_dtype):
    # 40 x 26 tiles, more than one per SM, so the default order is dynamic
    M, N, K = 40 * 128, 26 * 128, 256
    g = torch.Generator().manual_seed(24)
    a = torch.randn(M, K, generator=g)
    b = torch.randn(K, N, generator=g)
    a[-1] *= 300.0  # the last row block overflows against these columns
    b[:, -130:] *= 300.0
    a[:128] *= 300.0  # and the first
    a[1000] *= 300.0
    a, b = a.half().to(cuda), b.half().to(cuda)
    outs = run_all_orders(a, b, out_dtype)
    for c, _ in outs[1:]:
        assert torch.equal(c, outs[0][0])
    flags = check_redone(outs[0][0], outs[0][1], a, b, out_dtype)
    assert flags[-1, -1] and flags[0, -1] and not flags.all()


def test_one_cta_interleaves_main_and_redo_tiles(cuda):
    # an SM cap of 1: a single persistent CTA over 1024 tiles, its redo items
    # queued between main tiles as their flags come in
    M, N, K = 32 * 128, 32 * 128, 64
    g = torch.Generator().manual_seed(25)
    a = torch.randn(M, K, generator=g)
    b = torch.randn(K, N, generator=g)
    a[::300] *= 300.0
    b[:, ::700] *= 300.0
    a, b = a.half().to(cuda), b.half().to(cuda)
    with sm_limit(1):
        c1, ws1, c2, _ = both_modes(a, b, torch.float32)
    assert torch.equal(c1, c2)
    flags = check_redone(c1, ws1, a, b, torch.float32)
    assert flags.sum() > 20 and not flags.all()


def test_every_tile_flagged(cuda):
    # tests/test_f16acc.py:91-101 scaled up: every chunk of every tile overflows,
    # so every main tile queues a redo; the answer is exactly 100 everywhere
    x = torch.full((2048, 64), 100.0, device=cuda).half()
    w = torch.empty(2048, 64, device=cuda).half()
    w[:, :32] = 30.0
    w[:, 32:] = -30.0
    w[:, 63] = -29.0
    for c, ws in run_all_orders(x, w.t(), torch.float16):
        assert torch.all(c == 100.0)
        if ws is not None:
            assert tile_flags(ws, plan(x, w.t(), _lib.VARIANT_TCGEN05)).all()


def test_no_flags_same_as_separate(cuda):
    a = torch.randn(1024, 768, device=cuda).half()
    b = torch.randn(768, 896, device=cuda).half()
    c1, ws1, c2, _ = both_modes(a, b, torch.float16)
    assert torch.equal(c1, c2)
    assert not tile_flags(ws1, plan(a, b, _lib.VARIANT_TCGEN05)).any()


def test_redo_mode_knob_rejects_unknown_modes(cuda):
    lib = _lib.load()
    assert lib.f16acc_set_redo_mode(7) == _lib.ERR_INVALID_ARGUMENT
