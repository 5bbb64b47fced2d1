"""FP32 mode (`chunked=False`) with N >= 256 may run on 128x256 tiles
(f16acc_set_fp32_tiles: by a wave model, always, or never; an fp32 C is
staged in two column halves); every other FP32-mode call (N < 256, the redo
of flagged tiles) runs on 128x128 tiles.  Both issue the same K16 MMA sequence per output element, so
the results must be identical bit for bit (f16acc/kernel.py:50-51: one FP32
accumulator over all of K, then the cast), and within FP32 accumulation error
of an FP64 product."""

from contextlib import contextmanager

import pytest
import torch

from f16acc_b200 import _lib
from f16acc_b200.kernel import mm, mm_ex, plan, tile_flags

pytestmark = pytest.mark.gpu


@contextmanager
def fp32_tiles(mode):
    lib = _lib.load()
    prev = lib.f16acc_set_fp32_tiles(mode)
    assert prev >= 0
    try:
        yield
    finally:
        lib.f16acc_set_fp32_tiles(prev)

F32_TOL = 1e-5  # FP32 accumulation vs FP64, of max|ref|

SHAPES = [
    (256, 256, 64),      # one tile, one whole stage
    (300, 264, 520),     # ragged M and N (second tile 8 columns wide), K ends inside a stage
    (200, 1000, 776),    # N not a multiple of 256
    (1000, 512, 104),    # K shorter than two stages
    (640, 4096, 1536),   # full tiles, Qwen-like K
    (136, 264, 40),      # a few rows and columns past a tile, one partial stage
]


def operands(M, N, K, layout, cuda, seed):
    g = torch.Generator(device=cuda).manual_seed(seed)
    a = torch.randn(M, K, device=cuda, generator=g).half()
    if layout == "row_major":
        b = torch.randn(K, N, device=cuda, generator=g).half()
    else:  # nn.Linear weight [N, K] passed as w.t()
        b = torch.randn(N, K, device=cuda, generator=g).half().t()
    return a, b


@pytest.mark.parametrize("out_dtype", [torch.float16, torch.bfloat16, torch.float32], ids=str)
@pytest.mark.parametrize("layout", ["row_major", "w_t"])
@pytest.mark.parametrize("M,N,K", SHAPES, ids=[f"{m}x{n}x{k}" for m, n, k in SHAPES])
def test_wide_tiles_equal_the_128_wide_fp32_path(cuda, M, N, K, layout, out_dtype):
    a, b = operands(M, N, K, layout, cuda, seed=M + N + K)
    assert plan(a, b)["variant"] == _lib.VARIANT_TCGEN05  # strides TMA can take
    with fp32_tiles(_lib.FP32_TILES_WIDE):
        wide = mm(a, b, out_dtype, chunked=False)
    with fp32_tiles(_lib.FP32_TILES_NARROW):
        narrow_same_type = mm(a, b, out_dtype, chunked=False)
    narrow = mm(a, b, torch.float32, chunked=False)  # 128x128 tiles, fp32 C
    assert torch.equal(wide, narrow_same_type)
    assert torch.equal(wide, narrow.to(out_dtype))
    assert torch.equal(mm(a, b, out_dtype, chunked=False), wide)  # the default choice, whichever it is
    ref = a.double() @ b.double()
    err = (narrow.double() - ref).abs().max().item()
    assert err <= ref.abs().max().item() * F32_TOL


@pytest.mark.parametrize("out_dtype", [torch.float16, torch.float32], ids=str)
def test_wide_tiles_strided_output(cuda, out_dtype):
    """A column-major C leaves through the store warps' element-wise copy-out
    instead of TMA stores."""
    M, N, K = 384, 776, 320
    a, b = operands(M, N, K, "w_t", cuda, seed=9)
    out = torch.empty(N, M, device=cuda, dtype=out_dtype).t()
    with fp32_tiles(_lib.FP32_TILES_WIDE):
        c, _ = mm_ex(a, b, out_dtype, chunked=False, out=out)
    assert c.data_ptr() == out.data_ptr()
    with fp32_tiles(_lib.FP32_TILES_NARROW):
        narrow = mm(a, b, torch.float32, chunked=False)
    assert torch.equal(c, narrow.to(out_dtype))


def test_wide_tiles_bias(cuda):
    """The bias goes on in the epilogue of the wide tiles too, bit-equal to
    the product rounded to C's type and then y += b."""
    from f16acc_b200.kernel import mm_bias

    M, N, K = 256, 1032, 256
    a, b = operands(M, N, K, "w_t", cuda, seed=11)
    bias = torch.randn(N, device=cuda).half()
    for dt in (torch.float16, torch.float32):
        with fp32_tiles(_lib.FP32_TILES_WIDE):
            fused = mm_bias(a, b, bias, dt, chunked=False)
            ref = mm(a, b, dt, chunked=False)
        ref = (ref.float() + bias.float()).to(dt)
        assert torch.equal(fused, ref)


def test_wide_tiles_match_redone_tiles(cuda):
    """Redone tiles of a chunked call (128-wide FP32 recompute inside the
    chunked kernel) equal the wide-tile chunked=False output where the tiles
    were flagged."""
    n = 1024
    g = torch.Generator(device=cuda).manual_seed(3)
    a = torch.randn(n, n, device=cuda, generator=g)
    b = torch.randn(n, n, device=cuda, generator=g)
    a[5] *= 256  # row 5 x column 700: its FP16 chunk sums overflow
    b[:, 700] *= 256
    a, b = a.half(), b.half()
    c, ws = mm_ex(a, b, torch.float16)
    flags = tile_flags(ws, plan(a, b))
    assert flags.any()
    tm, tn = plan(a, b)["tile"]
    mask = flags.repeat_interleave(tm, 0).repeat_interleave(tn, 1)[:n, :n]
    with fp32_tiles(_lib.FP32_TILES_WIDE):
        c32 = mm(a, b, torch.float16, chunked=False)
    assert torch.equal(c[mask], c32[mask])

