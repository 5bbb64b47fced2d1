"""Tail split of the chunked tcgen05 main pass (f16acc_set_tail_split).

The tiles past the last full wave of the SMs run as S <= 4 units over
contiguous shares of K; the tile's last unit adds the units' FP32 partials in
K order.  The chunk semantics are unchanged (f16acc/kernel.py:44-49: every
32-long chunk accumulated in FP16 and added in FP32): only the association of
the FP32 chunk sum changes inside a split tile, so

- tiles that are not split are bit-identical with the split on and off;
- split tiles agree with the unsplit ones within FP32 rounding of the sum and
  with the oracle within the chunk bound of tests/helpers.py;
- flags are identical (f16acc/kernel.py:70-71), and flagged split tiles are
  redone over the whole of K in FP32 mode, bit-equal to chunked=False
  (f16acc/kernel.py:75-81);
- the result does not depend on which unit finishes last (repeat runs equal).
"""

from contextlib import contextmanager

import numpy as np
import pytest
import torch

from f16acc_b200 import _lib
from f16acc_b200.kernel import mm, mm_ex, plan, tile_flags, workspace_bytes
from oracle import oracle as O
from tests.helpers import chunk_ulp_bound_torch

pytestmark = pytest.mark.gpu

MIN_STAGES, MAX_SPLIT, MIN_SAVED = 6, 4, 20


@contextmanager
def tail_split(mode):
    lib = _lib.load()
    prev = lib.f16acc_set_tail_split(mode)
    assert prev >= 0
    try:
        yield
    finally:
        lib.f16acc_set_tail_split(prev)


def expected_split(M, N, K, sms):
    """(parts, split tiles) as the library plans them."""
    tiles = -(-M // 128) * -(-N // 128)
    nkb = -(-K // 64)
    r = tiles if tiles < sms else tiles % sms
    if r == 0:
        return 0, 0
    s = min(MAX_SPLIT, sms // r, nkb // MIN_STAGES)
    ok = s >= 2 and s * r <= 148 and nkb - nkb // s >= MIN_SAVED
    return (s, r) if ok else (0, 0)


def operands(M, N, K, layout, cuda, seed):
    g = torch.Generator(device=cuda).manual_seed(seed)
    a = (torch.randn(M, K, device=cuda, generator=g) * 4 / K ** 0.5).half()
    if layout == "w_t":
        b = (torch.randn(N, K, device=cuda, generator=g) * 4 / K ** 0.5).half().t()
    else:
        b = (torch.randn(K, N, device=cuda, generator=g) * 4 / K ** 0.5).half()
    return a, b


def tile_diff(x, y):
    """Per 128x128 tile: does any element differ."""
    d = (x != y).float()
    M, N = d.shape
    d = torch.nn.functional.pad(d, (0, -N % 128, 0, -M % 128))
    return d.reshape(d.shape[0] // 128, 128, d.shape[1] // 128, 128).amax(dim=(1, 3)) > 0


SHAPES = [
    (2048, 1536, 8960, "w_t"),   # Qwen down: 192 tiles, the last 44 in 3 parts
    (2048, 256, 4096, "w_t"),    # 32 tiles, every one in 4 parts
    (256, 128, 4096, "row_major"),  # 2 tiles in 4 parts
    (300, 264, 4000, "row_major"),  # ragged M and N, K ending inside a stage: 9 tiles in 4 parts
    (512, 512, 2752, "row_major"),  # 16 tiles in 4 parts of 10-11 stages
]


@pytest.mark.parametrize("M,N,K,layout", SHAPES, ids=[f"{m}x{n}x{k}" for m, n, k, _ in SHAPES])
def test_split_tiles_match_unsplit_and_oracle(cuda, M, N, K, layout):
    sms = torch.cuda.get_device_properties(cuda).multi_processor_count
    parts, split_tiles = expected_split(M, N, K, sms)
    assert parts >= 2, "shape chosen to split"
    a, b = operands(M, N, K, layout, cuda, seed=M + N + K)
    assert plan(a, b)["variant"] == _lib.VARIANT_TCGEN05
    with tail_split(_lib.TAIL_SPLIT_OFF):
        off, ws_off = mm_ex(a, b, torch.float32)
    with tail_split(_lib.TAIL_SPLIT_ON):
        on, ws_on = mm_ex(a, b, torch.float32)
        again = mm(a, b, torch.float32)
        on16 = mm(a, b, torch.float16)
    pl = plan(a, b)
    assert torch.equal(tile_flags(ws_on, pl), tile_flags(ws_off, pl))
    assert torch.equal(on, again)  # whichever unit adds the partials, the same sum
    assert torch.equal(on16, on.half())
    differ = tile_diff(on, off)
    assert int(differ.sum()) <= split_tiles  # only split tiles may move
    bound = chunk_ulp_bound_torch(a, b)
    assert ((on.double() - off.double()).abs() <= bound).all()
    # sampled rows against the CPU oracle (a row from every 128-row tile band)
    rows = torch.arange(0, M, 97)
    ref, _ = O.gemm_chunked(a[rows].cpu().numpy(), b.cpu().numpy(), round_every=16)
    err = np.abs(on[rows].double().cpu().numpy() - ref.astype(np.float64))
    assert (err <= bound[rows].cpu().numpy()).all()


@pytest.mark.parametrize("redo", ["inline", "separate"])
def test_flagged_split_tiles_are_redone_in_fp32(cuda, redo):
    """Overflowing chunk sums in split tiles flag the tile on the total; the
    tile is redone over all of K in FP32 (inside the kernel, or by the separate
    redo launch), bit-equal to chunked=False."""
    lib = _lib.load()
    prev = lib.f16acc_set_redo_mode(_lib.REDO_INLINE if redo == "inline" else _lib.REDO_SEPARATE)
    try:
        _flagged_split_tiles(cuda)
    finally:
        lib.f16acc_set_redo_mode(prev)


def _flagged_split_tiles(cuda):
    M, N, K = 2048, 1536, 4096
    g = torch.Generator(device=cuda).manual_seed(17)
    a = torch.randn(M, K, device=cuda, generator=g)
    b = torch.randn(K, N, device=cuda, generator=g)
    a[[5, 1900, 2047]] *= 300.0  # rows in the first and the last tile rows
    b[:, [3, 700, 1535]] *= 300.0
    a, b = a.half(), b.half()
    pl = plan(a, b)
    results = {}
    for mode in (_lib.TAIL_SPLIT_OFF, _lib.TAIL_SPLIT_ON):
        with tail_split(mode):
            c, ws = mm_ex(a, b, torch.float16)
            results[mode] = (c, tile_flags(ws, pl))
    (c_off, f_off), (c_on, f_on) = results[_lib.TAIL_SPLIT_OFF], results[_lib.TAIL_SPLIT_ON]
    assert f_on.any() and torch.equal(f_on, f_off)
    c32 = mm(a, b, torch.float16, chunked=False)
    tm, tn = pl["tile"]
    mask = f_on.repeat_interleave(tm, 0).repeat_interleave(tn, 1)[:M, :N]
    assert torch.equal(c_on[mask], c32[mask])
    assert torch.equal(c_on[mask], c_off[mask])


def test_flag_only_workspace_runs_unsplit(cuda):
    """A workspace that holds only the flags is accepted; the call then runs
    without the split, bit-equal to the split switched off."""
    M, N, K = 2048, 256, 4096
    a, b = operands(M, N, K, "w_t", cuda, seed=5)
    flag_bytes = (M // 128) * (N // 128) * 16
    assert workspace_bytes(M, N, K) > flag_bytes
    ws = torch.empty(flag_bytes, device=cuda, dtype=torch.uint8)
    c, _ = mm_ex(a, b, torch.float32, workspace=ws)
    with tail_split(_lib.TAIL_SPLIT_OFF):
        off = mm(a, b, torch.float32)
    assert torch.equal(c, off)
    small = torch.empty(flag_bytes - 16, device=cuda, dtype=torch.uint8)
    with pytest.raises(Exception):
        mm_ex(a, b, torch.float32, workspace=small)


@pytest.mark.parametrize("schedule", ["static", "dynamic"])
def test_split_under_both_tile_orders(cuda, schedule):
    """Qwen down at 2048 tokens has more units than SMs: the dynamic order
    hands the split units out as CTAs free up, the static one deals them round
    robin."""
    lib = _lib.load()
    M, N, K = 2048, 1536, 8960
    a, b = operands(M, N, K, "w_t", cuda, seed=23)
    with tail_split(_lib.TAIL_SPLIT_ON):
        ref = mm(a, b, torch.float32)
        prev = lib.f16acc_set_schedule(_lib.SCHEDULE_STATIC if schedule == "static" else _lib.SCHEDULE_DYNAMIC)
        try:
            c = mm(a, b, torch.float32)
        finally:
            lib.f16acc_set_schedule(prev)
    assert torch.equal(c, ref)


@pytest.mark.parametrize("out_dtype", [torch.float16, torch.bfloat16], ids=str)
def test_split_tiles_with_bias_and_narrow_outputs(cuda, out_dtype):
    """The last unit stages the total like a whole tile: the fused bias and the
    rounding to a 2-byte C match the unfused product plus y += b bit for bit."""
    from f16acc_b200.kernel import mm_bias

    M, N, K = 2048, 256, 4096
    a, b = operands(M, N, K, "w_t", cuda, seed=31)
    bias = torch.randn(N, device=cuda).half()
    with tail_split(_lib.TAIL_SPLIT_ON):
        full = mm(a, b, torch.float32)
        c = mm(a, b, out_dtype)
        fused = mm_bias(a, b, bias, out_dtype)
    assert torch.equal(c, full.to(out_dtype))
    assert torch.equal(fused, (c.float() + bias.float()).to(out_dtype))


@pytest.mark.parametrize("M,N,K,caps", [(2048, 256, 4096, (64, 100)), (2048, 1536, 4096, (128,))],
                         ids=["32_tiles", "192_tiles"])
def test_split_under_an_sm_cap(cuda, M, N, K, caps):
    """With f16acc_set_sm_limit the grid is a bounded persistent one in the
    static order, and the split plans for the capped SM count (32 tiles on 64
    SMs: 2 parts, on 100: 3; 192 tiles on 128: the last 64 in 2 parts, dealt
    round robin after the whole ones)."""
    lib = _lib.load()
    for cap in caps:
        assert expected_split(M, N, K, cap)[0] >= 2
    a, b = operands(M, N, K, "w_t", cuda, seed=41)
    with tail_split(_lib.TAIL_SPLIT_OFF):
        off = mm(a, b, torch.float32)
    bound = chunk_ulp_bound_torch(a, b)
    for cap in caps:
        prev = lib.f16acc_set_sm_limit(cap)
        try:
            with tail_split(_lib.TAIL_SPLIT_ON):
                c = mm(a, b, torch.float32)
                again = mm(a, b, torch.float32)
        finally:
            lib.f16acc_set_sm_limit(prev)
        assert torch.equal(c, again)
        assert ((c.double() - off.double()).abs() <= bound).all()
