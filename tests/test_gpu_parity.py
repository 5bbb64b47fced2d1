"""Parity of the CUDA kernels (through the C ABI) with the CPU oracle and the
reference's golden outputs.

Tolerances.  Within one 32-long chunk the FP16 rounding order is hardware
defined (the reference leaves it to Triton), so two correct chunked results
may differ by a rounding of each chunk sum: the bound is 2 FP16 ulps of every
chunk value plus FP32 rounding of the running sum (tests/helpers.py).  Tile
flags, the overflow known answer, and redone tiles against the kernel's own
FP32-accumulate output are exact.  FP32-accumulate results (hardware order
of FP32 additions): F32_TOL = 1e-5 of max|ref|.
"""

import os

import numpy as np
import pytest
import torch

import f16acc_b200 as f16acc
from f16acc_b200 import _lib
from f16acc_b200.kernel import mm_ex, plan, tile_flags, device_status
from oracle import oracle as O
from tests.helpers import chunk_ulp_bound, rel

pytestmark = pytest.mark.gpu

VARIANTS = [_lib.VARIANT_TCGEN05, _lib.VARIANT_MMA_SYNC]
VNAMES = {_lib.VARIANT_TCGEN05: "tcgen05", _lib.VARIANT_MMA_SYNC: "mma_sync"}
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "reference_cases.npz")
F32_TOL = 1e-5


def padded(x: torch.Tensor, mult: int = 8) -> torch.Tensor:
    """Same values, rows padded to a multiple of `mult` elements (TMA needs
    16-byte aligned row strides); returns a view of the padded buffer."""
    rows, cols = x.shape
    buf = torch.zeros(rows, (cols + mult - 1) // mult * mult, dtype=x.dtype, device=x.device)
    buf[:, :cols] = x
    return buf[:, :cols]


def tma_ready(a, b):
    """Operands laid out so the tcgen05 variant accepts them: A K-contiguous,
    B either N-contiguous or K-contiguous (a transposed view), rows aligned."""
    if b.stride(0) == 1 and b.stride(1) != 1:  # K-contiguous B (w.t())
        return padded(a), padded(b.t()).t()
    return padded(a), padded(b)


def np16(t):
    return t.detach().cpu().numpy()


def run(a, b, variant, out_dtype=torch.float32, chunked=True):
    if variant == _lib.VARIANT_TCGEN05:
        a, b = tma_ready(a, b)
    c, ws = mm_ex(a, b, out_dtype, chunked, variant=variant)
    return c, ws, a, b


def check_chunked(c, a, b, ulps=2.0):
    a_np, b_np = np16(a), np16(b)
    ref, _ = O.gemm_chunked(a_np, b_np, round_every=16)
    bound = chunk_ulp_bound(a_np, b_np, ulps=ulps)
    cc = c.double().cpu().numpy()
    if c.dtype != torch.float32:
        bound = bound + np.abs(ref) * 2.0 ** -7 if c.dtype == torch.bfloat16 else bound + np.abs(ref) * 2.0 ** -10
    err = np.abs(cc - ref)
    assert np.isfinite(cc).all()
    assert (err <= bound).all(), f"max err {err.max()} (bound there {bound.flat[err.argmax()]})"


# ---------------------------------------------------------------- golden fixtures

def _golden():
    z = np.load(GOLDEN)
    names = sorted({k.split("/")[0] for k in z.files})
    return [(n, {k.split("/", 1)[1]: z[k] for k in z.files if k.startswith(n + "/")}) for n in names]


@pytest.mark.parametrize("variant", VARIANTS, ids=VNAMES.get)
@pytest.mark.parametrize("name,d", _golden(), ids=[n for n, _ in _golden()])
def test_golden_reference_outputs(cuda, variant, name, d):
    a = torch.from_numpy(d["a"]).to(cuda)
    b = torch.from_numpy(d["b"]).to(cuda) if "b" in d else torch.from_numpy(d["b_t"]).to(cuda).t()
    out_dtype = torch.float16 if str(d["out"]) == "torch.float16" else torch.float32
    chunked = bool(d["chunked"])
    c, ws, a2, b2 = run(a, b, variant, out_dtype, chunked)
    ref = d["c"].astype(np.float64)
    cc = c.double().cpu().numpy()
    if "overflow_kat" in name:
        assert (cc == 100.0).all()
        return
    if not chunked:
        assert np.abs(cc - ref).max() <= np.abs(ref).max() * F32_TOL
        return
    bound = chunk_ulp_bound(d["a"], np16(b), ulps=2.0)
    if out_dtype == torch.float16:
        bound = bound + 2 * np.maximum(np.abs(ref) * 2.0 ** -11, 2.0 ** -25)
    # tiles the reference redid (its 64x64 grid) hold FP32-accumulate values
    rflags = d["flags"].reshape((d["a"].shape[0] + 63) // 64, -1).astype(bool)
    redone = np.repeat(np.repeat(rflags, 64, 0), 64, 1)[: ref.shape[0], : ref.shape[1]]
    ours_flags = tile_flags(ws, plan(a2, b2, variant)).cpu().numpy()
    pm, pn = plan(a2, b2, variant)["tile"]
    ours_redone = np.repeat(np.repeat(ours_flags, pm, 0), pn, 1)[: ref.shape[0], : ref.shape[1]]
    either = redone | ours_redone
    f32 = O.gemm_f32acc(d["a"], np16(b)).astype(np.float64)
    # where exactly one side redid a tile, values are compared to the FP32 product instead
    both_ok = np.where(either, np.abs(cc - f32) <= np.abs(f32).max() * F32_TOL, np.abs(cc - ref) <= bound)
    assert both_ok.all(), float(np.abs(cc - ref).max())


# ---------------------------------------------------------------- configs and shapes

@pytest.mark.parametrize("variant", VARIANTS, ids=VNAMES.get)
def test_config1_512_uniform_fp32_out(cuda, variant):
    # 512^3, A,B ~ U[-1,1] seed 0, fp32 out; within 1e-3 of FP64
    g = torch.Generator().manual_seed(0)
    a = (torch.rand(512, 512, generator=g) * 2 - 1).half().to(cuda)
    b = (torch.rand(512, 512, generator=g) * 2 - 1).half().to(cuda)
    c, *_ = run(a, b, variant)
    assert rel(c.cpu().numpy(), O.gemm_f64(np16(a), np16(b))) < 1e-3
    check_chunked(c, a, b)


@pytest.mark.parametrize("variant", VARIANTS, ids=VNAMES.get)
@pytest.mark.parametrize("K", [1, 8, 15, 16, 17, 31, 32, 33, 63, 64, 65, 96, 100, 200, 777])
def test_k_tails(cuda, variant, K):
    g = torch.Generator().manual_seed(K)
    a = torch.randn(200, K, generator=g).half().to(cuda)
    b = torch.randn(K, 136, generator=g).half().to(cuda)
    c, *_ = run(a, b, variant)
    check_chunked(c, a, b)


@pytest.mark.parametrize("variant", VARIANTS, ids=VNAMES.get)
@pytest.mark.parametrize("M,N", [(1, 1), (1, 300), (129, 1), (127, 129), (384, 640), (1000, 1234)])
def test_ragged_m_n(cuda, variant, M, N):
    g = torch.Generator().manual_seed(M * 7 + N)
    a = torch.randn(M, 96, generator=g).half().to(cuda)
    b = torch.randn(96, N, generator=g).half().to(cuda)
    c, *_ = run(a, b, variant)
    check_chunked(c, a, b)


@pytest.mark.parametrize("variant", VARIANTS, ids=VNAMES.get)
@pytest.mark.parametrize("out_dtype", [torch.float16, torch.float32, torch.bfloat16], ids=str)
@pytest.mark.parametrize("layout", ["row_major", "w_t"])
def test_layouts_and_output_types(cuda, variant, out_dtype, layout):
    g = torch.Generator().manual_seed(11)
    a = torch.randn(256, 320, generator=g).half().to(cuda)
    if layout == "row_major":
        b = torch.randn(320, 384, generator=g).half().to(cuda)
    else:
        b = torch.randn(384, 320, generator=g).half().to(cuda).t()
    c, *_ = run(a, b, variant, out_dtype)
    assert c.dtype == out_dtype
    check_chunked(c, a, b)


def test_generic_strides_take_the_mma_sync_path(cuda):
    g = torch.Generator().manual_seed(5)
    big_a = torch.randn(300, 500, generator=g).half().to(cuda)
    big_b = torch.randn(400, 900, generator=g).half().to(cuda)
    cases = [
        (big_a[::2, 1:200:1], big_b[:199, ::3]),          # odd offsets, N stride 3
        (big_a.t()[:250, :150], big_b[:150, 5:133]),       # M-contiguous A
        (big_a[:100, :77], big_b.t()[:77, :260]),          # K=77 unaligned, K-contiguous B
    ]
    for a, b in cases:
        assert plan(a, b)["variant"] == _lib.VARIANT_MMA_SYNC
        c = f16acc.mm(a, b, torch.float32)
        check_chunked(c, a, b)


def test_strided_outputs_through_the_c_abi(cuda):
    g = torch.Generator().manual_seed(6)
    a = torch.randn(200, 128, generator=g).half().to(cuda)
    b = torch.randn(128, 160, generator=g).half().to(cuda)
    ref, _ = mm_ex(a, b, torch.float32)
    for variant in VARIANTS:
        wide = torch.full((200, 300), -7.0, device=cuda)
        out = wide[:, 50:210]
        mm_ex(a, b, torch.float32, variant=variant, out=out)
        if variant == plan(a, b)["variant"]:
            assert torch.equal(out, ref)  # same kernel as the contiguous-output call
        assert (wide[:, :50] == -7).all() and (wide[:, 210:] == -7).all()
        check_chunked(out, a, b)
        colmajor = torch.empty(160, 200, device=cuda).t()
        mm_ex(a, b, torch.float32, variant=variant, out=colmajor)
        check_chunked(colmajor, a, b)


@pytest.mark.parametrize("out_dtype", [torch.float16, torch.bfloat16, torch.float32], ids=str)
def test_padded_row_outputs_take_tma_stores(cuda, out_dtype):
    # C is a 16-byte aligned column window of a wider buffer: the tcgen05 kernel
    # writes it with TMA bulk stores through a tensor map of row stride 320
    # elements.  M and N are not tile multiples, so the boxes are clipped at
    # both edges; nothing outside the window may change.
    g = torch.Generator().manual_seed(16)
    a = torch.randn(200, 256, generator=g).half().to(cuda)
    b = torch.randn(256, 168, generator=g).half().to(cuda)
    ref, _ = mm_ex(a, b, out_dtype)
    assert plan(a, b)["variant"] == _lib.VARIANT_TCGEN05
    wide = torch.full((200, 320), -7.0, device=cuda, dtype=out_dtype)
    col0 = 64  # 128 or 256 bytes into each row
    out = wide[:, col0:col0 + 168]
    mm_ex(a, b, out_dtype, out=out)
    assert torch.equal(out, ref)
    assert (wide[:, :col0] == -7).all() and (wide[:, col0 + 168:] == -7).all()
    check_chunked(out, a, b)


@pytest.mark.parametrize("variant", VARIANTS, ids=VNAMES.get)
def test_fp32_accumulate_mode(cuda, variant):
    g = torch.Generator().manual_seed(7)
    a = torch.randn(300, 500, generator=g).half().to(cuda)
    b = torch.randn(500, 260, generator=g).half().to(cuda)
    c, *_ = run(a, b, variant, chunked=False)
    ref = O.gemm_f64(np16(a), np16(b))
    assert np.abs(c.double().cpu().numpy() - ref).max() <= np.abs(ref).max() * F32_TOL


def test_empty_shapes(cuda):
    a = torch.randn(256, 0, device=cuda).half()
    b = torch.randn(0, 48, device=cuda).half()
    for dt in (torch.float16, torch.float32):
        c = f16acc.mm(a, b, dt)
        assert c.shape == (256, 48) and (c == 0).all()
    assert f16acc.mm(torch.randn(0, 64, device=cuda).half(), torch.randn(64, 5, device=cuda).half()).shape == (0, 5)
    assert f16acc.mm(torch.randn(7, 64, device=cuda).half(), torch.randn(64, 0, device=cuda).half()).shape == (7, 0)


# ---------------------------------------------------------------- overflow, flags and redo

def stress(M, N, K, seed, scale=256.0, frac=0.01):
    """Config-4 style: N(0,1) operands with ~1% of A rows and B columns scaled
    so 32-long FP16 chunk sums in the crossed tiles exceed 65504."""
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(M, K, generator=g)
    b = torch.randn(K, N, generator=g)
    rows = torch.randperm(M, generator=g)[: max(1, int(M * frac))]
    cols = torch.randperm(N, generator=g)[: max(1, int(N * frac))]
    a[rows] *= scale
    b[:, cols] *= scale
    return a.half(), b.half()


@pytest.mark.parametrize("variant", VARIANTS, ids=VNAMES.get)
@pytest.mark.parametrize("layout", ["row_major", "w_t"])
def test_redo_tiles_equal_fp32_path_bitwise(cuda, variant, layout):
    a, b = stress(512, 640, 384, seed=3)
    a, b = a.to(cuda), b.to(cuda)
    if layout == "w_t":
        b = b.t().contiguous().t()
    c, ws, a2, b2 = run(a, b, variant)
    c32, *_ = run(a, b, variant, chunked=False)
    pl = plan(a2, b2, variant)
    flags = tile_flags(ws, pl).cpu().numpy()
    # flags equal the oracle's at this tile shape
    _, oflags = O.gemm_chunked(np16(a), np16(b), round_every=16, tile=pl["tile"], redo=False)
    assert flags.any() and not flags.all()
    np.testing.assert_array_equal(flags, oflags.astype(bool))
    tm, tn = pl["tile"]
    cc, c32c = c.cpu(), c32.cpu()
    for i, j in zip(*np.nonzero(flags)):
        sl = (slice(i * tm, (i + 1) * tm), slice(j * tn, (j + 1) * tn))
        assert torch.equal(cc[sl], c32c[sl]), f"redone tile {(i, j)} differs from the FP32-accumulate output"
    assert torch.isfinite(c).all()
    # unflagged tiles are chunked results
    mask = np.repeat(np.repeat(flags, tm, 0), tn, 1)[: c.shape[0], : c.shape[1]]
    ref, _ = O.gemm_chunked(np16(a), np16(b), round_every=16)
    bound = chunk_ulp_bound(np16(a), np16(b))
    err = np.abs(cc.double().numpy() - ref)
    assert (err[~mask] <= bound[~mask]).all()


@pytest.mark.parametrize("variant", VARIANTS, ids=VNAMES.get)
@pytest.mark.parametrize("layout", ["row_major", "w_t"])
def test_overflow_known_answer(cuda, variant, layout):
    # tests/test_f16acc.py:91-101 through mm directly: every chunk overflows, the result is exactly 100
    x = torch.full((256, 64), 100.0, device=cuda).half()
    w = torch.empty(128, 64, device=cuda).half()
    w[:, :32] = 30.0
    w[:, 32:] = -30.0
    w[:, 63] = -29.0
    b = w.t() if layout == "w_t" else w.t().contiguous()
    c, ws, a2, b2 = run(x, b, variant, torch.float16)
    assert torch.all(c == 100.0)
    assert tile_flags(ws, plan(a2, b2, variant)).all()


def test_no_flags_on_benign_inputs(cuda):
    a = torch.randn(512, 1024, device=cuda).half()
    b = torch.randn(1024, 512, device=cuda).half()
    for variant in VARIANTS:
        c, ws, a2, b2 = run(a, b, variant)
        assert not tile_flags(ws, plan(a2, b2, variant)).any()


def test_deterministic(cuda):
    a = torch.randn(640, 768, device=cuda).half()
    b = torch.randn(768, 896, device=cuda).half()
    for variant in VARIANTS:
        c1, *_ = run(a, b, variant)
        c2, *_ = run(a, b, variant)
        assert torch.equal(c1, c2)


# ---------------------------------------------------------------- full-size configs (size-independent properties)

@pytest.mark.parametrize("layout", ["row_major", "w_t"])
@pytest.mark.parametrize("out_dtype", [torch.float16, torch.float32], ids=str)
def test_config2_4096_accuracy(cuda, layout, out_dtype):
    # N(0,1)/sqrt(K)*4 seed 1; north star: max rel err <= 1e-3 vs FP64
    g = torch.Generator(device=cuda).manual_seed(1)
    n = 4096
    a = (torch.randn(n, n, device=cuda, generator=g) / n ** 0.5 * 4).half()
    b = (torch.randn(n, n, device=cuda, generator=g) / n ** 0.5 * 4).half()
    if layout == "w_t":
        b = b.t().contiguous().t()
    assert plan(a, b)["variant"] == _lib.VARIANT_TCGEN05
    ref = a.double() @ b.double()
    c = f16acc.mm(a, b, out_dtype)
    r = ((c.double() - ref).abs().max() / ref.abs().max()).item()
    assert r <= 1e-3
    # the mma.sync variant computes the same chunked product
    c2, _ = mm_ex(a, b, out_dtype, variant=_lib.VARIANT_MMA_SYNC)
    r2 = ((c2.double() - ref).abs().max() / ref.abs().max()).item()
    assert r2 <= 1e-3


@pytest.mark.parametrize("out_dtype", [torch.float16, torch.float32], ids=str)
def test_config4_overflow_stress_4096(cuda, out_dtype):
    # N(0,1) seed 3, 1% of A rows and B cols x64
    a, b = stress(4096, 4096, 4096, seed=3, scale=64.0)
    a, b = a.to(cuda), b.to(cuda)
    c, ws = mm_ex(a, b, out_dtype)
    c32, _ = mm_ex(a, b, out_dtype, chunked=False)
    pl = plan(a, b)
    flags = tile_flags(ws, pl)
    assert flags.any()
    tm, tn = pl["tile"]
    mask = flags.repeat_interleave(tm, 0).repeat_interleave(tn, 1)[: c.shape[0], : c.shape[1]]
    assert torch.equal(c[mask], c32[mask])  # redone tiles == the FP32-accumulate path, bit for bit
    ref = a.double() @ b.double()
    # an fp16 store of |C| > 65504 is inf, exactly as the reference's cast (kernel.py:59); never NaN
    fits = ref.abs() < 65000 if out_dtype == torch.float16 else torch.ones_like(ref, dtype=torch.bool)
    assert torch.isfinite(c[fits]).all() and not torch.isnan(c).any()
    assert ((c.double()[fits] - ref[fits]).abs().max() / ref.abs().max()).item() < 1e-3


def test_device_status_clean(cuda):
    assert device_status(0, reset=True) == 0


# ---------------------------------------------------------------- hardware rounding inside a chunk

@pytest.mark.parametrize("dist", ["normal", "uniform", "wide"])
def test_chunk_rounding_matches_round_every_16(cuda, dist):
    """K = 32, so C is one chunk value converted exactly to FP32.  Both
    variants give bit-identical chunk values, and they equal the oracle's
    round-after-each-K=16 emulation in (almost) every element."""
    g = torch.Generator().manual_seed(1)
    if dist == "normal":
        a, b = torch.randn(512, 32, generator=g), torch.randn(32, 512, generator=g)
    elif dist == "uniform":
        a, b = torch.rand(512, 32, generator=g) * 2 - 1, torch.rand(32, 512, generator=g) * 2 - 1
    else:
        a = torch.randn(512, 32, generator=g) * torch.exp2(torch.randint(-6, 6, (512, 32), generator=g).float())
        b = torch.randn(32, 512, generator=g)
    a, b = a.half(), b.half()
    r16, _ = O.gemm_chunked(a.numpy(), b.numpy(), round_every=16)
    r32, _ = O.gemm_chunked(a.numpy(), b.numpy(), round_every=32)
    outs = [mm_ex(a.to(cuda), b.to(cuda), torch.float32, variant=v)[0].cpu().numpy() for v in VARIANTS]
    assert np.array_equal(outs[0], outs[1])
    eq16 = float((outs[0] == r16).mean())
    eq32 = float((outs[0] == r32).mean())
    print(f"\n{dist}: equal to round_every=16 {eq16:.5f}, to round_every=32 {eq32:.5f}")
    assert eq16 > 0.999 and eq16 > eq32
