"""The few-row kernel (F16ACC_VARIANT_SKINNY, the automatic choice for M <= 64, M <= 32 when N > 32768):
parity with the CPU oracle, flags, the redo, bias and layouts.

Its chunk values are the same m16n8k16 FP16-accumulate results as the other
kernels'; the FP32 sum over chunks is formed per K range of the CTA cluster
and the partials added after, an FP32 rounding difference that the chunk
bound (tests/helpers.py) already allows for.
"""

import numpy as np
import pytest
import torch

import f16acc_b200 as f16acc
from f16acc_b200 import _lib
from f16acc_b200.kernel import mm_bias, mm_ex, plan, tile_flags
from oracle import oracle as O
from tests.helpers import chunk_ulp_bound, rel
from tests.test_gpu_parity import F32_TOL, np16

pytestmark = pytest.mark.gpu
SK = _lib.VARIANT_SKINNY


def operands(M, N, K, seed, device, layout="w_t", scale=1.0):
    g = torch.Generator().manual_seed(seed)
    a = (torch.randn(M, K, generator=g) * scale).half().to(device)
    w = (torch.randn(N, K, generator=g) * scale).half().to(device)
    b = w.t() if layout == "w_t" else w.t().contiguous()
    return a, b


def check_chunked(c, a, b):
    ref, _ = O.gemm_chunked(np16(a), np16(b), round_every=16)
    bound = chunk_ulp_bound(np16(a), np16(b))
    err = np.abs(c.double().cpu().numpy() - ref)
    assert (err <= bound).all(), f"max excess {(err - bound).max()}"


@pytest.mark.parametrize("M", [1, 7, 16, 17, 33, 64])
@pytest.mark.parametrize("layout", ["w_t", "row_major"])
def test_chunked_parity_with_oracle(cuda, M, layout):
    a, b = operands(M, 304, 1000, seed=M, device=cuda, layout=layout)  # 16-byte aligned rows either way
    assert plan(a, b)["variant"] == SK
    c, _ = mm_ex(a, b, torch.float32)
    check_chunked(c, a, b)


@pytest.mark.parametrize("K", [8, 16, 40, 64, 200, 4104])
@pytest.mark.parametrize("N", [8, 77, 128, 264])
def test_k_and_n_tails(cuda, K, N):
    a, b = operands(5, N, K, seed=K + N, device=cuda)
    c, _ = mm_ex(a, b, torch.float32, variant=SK)
    check_chunked(c, a, b)
    c32, _ = mm_ex(a, b, torch.float32, chunked=False, variant=SK)
    ref = O.gemm_f64(np16(a), np16(b))
    assert np.abs(c32.double().cpu().numpy() - ref).max() <= np.abs(ref).max() * F32_TOL + 1e-6


def test_automatic_choice(cuda):
    for M, want in ((1, SK), (64, SK), (65, _lib.VARIANT_TCGEN05)):
        a, b = operands(M, 256, 256, seed=1, device=cuda)
        assert plan(a, b)["variant"] == want
    for M, want in ((32, SK), (33, _lib.VARIANT_TCGEN05)):  # very wide products
        a, b = operands(M, 40000, 64, seed=1, device=cuda)
        assert plan(a, b)["variant"] == want
    a, b = operands(16, 256, 256, seed=1, device=cuda)
    assert plan(a[:, 1:], b[1:])["variant"] != SK  # unaligned rows: not a cp.async operand


@pytest.mark.parametrize("out_dtype", [torch.float16, torch.float32, torch.bfloat16], ids=str)
def test_output_types_and_accuracy(cuda, out_dtype):
    a, b = operands(16, 4096, 4096, seed=3, device=cuda, scale=4.0 / 64)
    c = f16acc.mm(a, b, out_dtype)
    # the north star's 1e-3 vs FP64; a bf16 output alone rounds by up to 2^-9 of |C|
    bar = 2.0 ** -8 if out_dtype == torch.bfloat16 else 1e-3
    assert rel(c.double().cpu(), O.gemm_f64(np16(a), np16(b))) < bar


def stress_small(M, N, K, seed, device):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(M, K, generator=g)
    w = torch.randn(N, K, generator=g)
    a[M // 2] *= 300.0
    w[100:120] *= 300.0  # tile 0 (columns 0-127) overflows in row M // 2
    w[700:705] *= 300.0  # and tile 5
    return a.half().to(device), w.half().to(device).t()


@pytest.mark.parametrize("M", [16, 48])
def test_flags_and_redo(cuda, M):
    a, b = stress_small(M, 1000, 512, seed=M, device=cuda)
    c, ws = mm_ex(a, b, torch.float32, variant=SK)
    pl = plan(a, b, SK)
    flags = tile_flags(ws, pl).cpu().numpy()
    _, oflags = O.gemm_chunked(np16(a), np16(b), round_every=16, tile=pl["tile"], redo=False)
    np.testing.assert_array_equal(flags, oflags.astype(bool))
    assert flags[0, 0] and flags[0, 5] and flags.sum() == 2
    c32, _ = mm_ex(a, b, torch.float32, chunked=False, variant=SK)
    tn = pl["tile"][1]
    for j in np.nonzero(flags[0])[0]:
        assert torch.equal(c[:, j * tn:(j + 1) * tn], c32[:, j * tn:(j + 1) * tn])
    mask = np.repeat(flags[0], tn)[: c.shape[1]]
    ref, _ = O.gemm_chunked(np16(a), np16(b), round_every=16)
    bound = chunk_ulp_bound(np16(a), np16(b))
    err = np.abs(c.double().cpu().numpy() - ref)
    assert (err[:, ~mask] <= bound[:, ~mask]).all()
    # the same bits with the redo as a second launch
    lib = _lib.load()
    prev = lib.f16acc_set_redo_mode(_lib.REDO_SEPARATE)
    try:
        c2, _ = mm_ex(a, b, torch.float32, variant=SK)
    finally:
        lib.f16acc_set_redo_mode(prev)
    assert torch.equal(c, c2)


@pytest.mark.parametrize("M", [1, 17, 32])
def test_wide_launch_shallow_ring(cuda, M):
    # more single-CTA column tiles than one wave holds (N = 38017: 298 tiles,
    # the last 1 column wide): the 3-stage ring; parity with the oracle, flags
    # and the in-kernel redo of two overflowing tiles
    N, K = 38017, 200
    g = torch.Generator().manual_seed(M)
    a = torch.randn(M, K, generator=g)
    w = torch.randn(N, K, generator=g)
    a[0] *= 300.0
    w[5] *= 300.0       # tile 0
    w[38000] *= 300.0   # tile 296
    a, w = a.half().to(cuda), w.half().to(cuda)
    b = w.t()
    assert plan(a, b)["variant"] == SK
    c, ws = mm_ex(a, b, torch.float32)
    pl = plan(a, b, SK)
    flags = tile_flags(ws, pl).cpu().numpy()
    _, oflags = O.gemm_chunked(np16(a), np16(b), round_every=16, tile=pl["tile"], redo=False)
    np.testing.assert_array_equal(flags, oflags.astype(bool))
    assert flags[0, 0] and flags[0, 296] and flags.sum() == 2
    c32, _ = mm_ex(a, b, torch.float32, chunked=False)
    tn = pl["tile"][1]
    mask = np.repeat(flags[0], tn)[:N]
    assert torch.equal(c[:, torch.from_numpy(mask).to(cuda)], c32[:, torch.from_numpy(mask).to(cuda)])
    ref, _ = O.gemm_chunked(np16(a), np16(b), round_every=16)
    bound = chunk_ulp_bound(np16(a), np16(b))
    err = np.abs(c.double().cpu().numpy() - ref)
    assert (err[:, ~mask] <= bound[:, ~mask]).all()


def test_overflow_known_answer(cuda):
    # tests/test_f16acc.py:91-101 with 16 rows: every chunk overflows, the answer is exactly 100
    x = torch.full((16, 64), 100.0, device=cuda).half()
    w = torch.empty(128, 64, device=cuda).half()
    w[:, :32] = 30.0
    w[:, 32:] = -30.0
    w[:, 63] = -29.0
    c, ws = mm_ex(x, w.t(), torch.float16, variant=SK)
    assert torch.all(c == 100.0)
    assert tile_flags(ws, plan(x, w.t(), SK)).all()


@pytest.mark.parametrize("out_dtype", [torch.float16, torch.float32], ids=str)
def test_bias_equals_mm_then_add(cuda, out_dtype):
    a, b = operands(9, 520, 384, seed=7, device=cuda)
    bias = torch.randn(520, device=cuda).half()
    c = mm_bias(a, b, bias, out_dtype)
    y = f16acc.mm(a, b, out_dtype)
    y += bias
    assert torch.equal(c, y)


def test_strided_output(cuda):
    a, b = operands(20, 200, 256, seed=8, device=cuda)
    ref, _ = mm_ex(a, b, torch.float32, variant=SK)
    colmajor = torch.empty(200, 20, device=cuda).t()
    mm_ex(a, b, torch.float32, variant=SK, out=colmajor)
    assert torch.equal(colmajor, ref)


def test_deterministic(cuda):
    a, b = operands(32, 3000, 2048, seed=9, device=cuda)
    c1, _ = mm_ex(a, b, torch.float16, variant=SK)
    c2, _ = mm_ex(a, b, torch.float16, variant=SK)
    assert torch.equal(c1, c2)


def test_device_status_clean(cuda):
    assert _lib.load().f16acc_device_status(0, 1) == 0
