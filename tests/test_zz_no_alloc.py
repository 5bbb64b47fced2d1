"""f16acc_gemm_noalloc: the entry point for callers that cannot allocate
device memory (a plain C / FFI program with raw pointers and no device
allocator, or a loop that must not call cudaMalloc).  It keeps the per-tile
overflow flags in a fixed array inside the library instead of a caller
workspace.

Called through the C ABI, its output must equal the allocating entry point's
(f16acc_gemm with a workspace) on two calls in a row; the chunked inputs
overflow FP16 in some tiles, so the flag array and the redo pass are
exercised, and the second call runs on whatever the first left in the shared
array.  The file name sorts last so a run that stops at the first failure has
already run every other test; it also passes alone in a fresh process.
"""

import pytest
import torch

from f16acc_b200 import _lib

pytestmark = pytest.mark.gpu


def _stress(M, N, K, seed):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(M, K, generator=g)
    b = torch.randn(K, N, generator=g)
    a[torch.randperm(M, generator=g)[: M // 64]] *= 256.0  # some 32-long chunk sums overflow FP16
    b[:, torch.randperm(N, generator=g)[: N // 64]] *= 256.0
    return a.half(), b.half()


def _reference(lib, a, b, out_dtype, chunked):
    M, K = a.shape
    N = b.shape[1]
    c = torch.empty(M, N, device=a.device, dtype=out_dtype)
    ws = torch.empty(lib.f16acc_workspace_bytes(M, N, K), device=a.device, dtype=torch.uint8)
    stream = torch.cuda.current_stream(a.device).cuda_stream
    code = {torch.float16: _lib.OUT_F16, torch.float32: _lib.OUT_F32}[out_dtype]
    rc = lib.f16acc_gemm(a.data_ptr(), a.stride(0), a.stride(1), b.data_ptr(), b.stride(0), b.stride(1),
                         c.data_ptr(), c.stride(0), c.stride(1), code, M, N, K, 1 if chunked else 0,
                         ws.data_ptr(), ws.numel(), a.device.index or 0, stream)
    assert rc == _lib.OK, _lib.strerror(rc)
    return c


def _flagged_tiles(lib, a, b):
    """Tiles the allocating entry point flags for these operands (its own,
    freshly allocated workspace)."""
    M, K = a.shape
    N = b.shape[1]
    c = torch.empty(M, N, device=a.device, dtype=torch.float32)
    ws = torch.empty(lib.f16acc_workspace_bytes(M, N, K), device=a.device, dtype=torch.uint8)
    rc = lib.f16acc_gemm(a.data_ptr(), a.stride(0), a.stride(1), b.data_ptr(), b.stride(0), b.stride(1),
                         c.data_ptr(), c.stride(0), c.stride(1), _lib.OUT_F32, M, N, K, 1, ws.data_ptr(),
                         ws.numel(), a.device.index or 0, torch.cuda.current_stream(a.device).cuda_stream)
    assert rc == _lib.OK
    return int(ws.view(-1, 16).ne(0).any(dim=1).sum())


def _noalloc(lib, a, b, out_dtype, chunked, out=None):
    M, K = a.shape
    N = b.shape[1]
    c = out if out is not None else torch.empty(M, N, device=a.device, dtype=out_dtype)
    stream = torch.cuda.current_stream(a.device).cuda_stream
    code = {torch.float16: _lib.OUT_F16, torch.float32: _lib.OUT_F32}[out_dtype]
    rc = lib.f16acc_gemm_noalloc(a.data_ptr(), a.stride(0), a.stride(1), b.data_ptr(), b.stride(0), b.stride(1),
                                 c.data_ptr(), c.stride(0), c.stride(1), code, M, N, K, 1 if chunked else 0,
                                 a.device.index or 0, stream)
    return rc, c


@pytest.mark.parametrize("layout", ["row_major", "w_t", "unaligned"])
def test_noalloc_matches_allocating_entry_point_twice(cuda, layout):
    lib = _lib.load()
    a, b = _stress(512, 640, 384, seed=11)
    a, b = a.to(cuda), b.to(cuda)
    if layout == "w_t":
        b = b.t().contiguous().t()  # nn.Linear weight layout: K-contiguous B (tcgen05 path)
    elif layout == "unaligned":
        a = torch.nn.functional.pad(a, (0, 3))[:, :384]  # row stride 387: the mma.sync path
    for out_dtype in (torch.float32, torch.float16):
        ref = _reference(lib, a, b, out_dtype, True)
        torch.cuda.synchronize()
        assert torch.isnan(ref).sum() == 0
        for _ in range(2):  # the second call reuses the shared flag array as the first left it
            rc, c = _noalloc(lib, a, b, out_dtype, True)
            assert rc == _lib.OK, _lib.strerror(rc)
            torch.cuda.synchronize()
            assert torch.equal(c, ref)


def test_noalloc_fp32_accumulate_and_other_shapes(cuda):
    lib = _lib.load()
    g = torch.Generator().manual_seed(5)
    for M, N, K in ((300, 260, 500), (128, 128, 32), (1000, 1234, 777)):
        a = torch.randn(M, K, generator=g).half().to(cuda)
        b = torch.randn(K, N, generator=g).half().to(cuda)
        for chunked in (True, False):
            ref = _reference(lib, a, b, torch.float32, chunked)
            for _ in range(2):
                rc, c = _noalloc(lib, a, b, torch.float32, chunked)
                assert rc == _lib.OK
                torch.cuda.synchronize()
                assert torch.equal(c, ref)


@pytest.mark.parametrize("redo", ["inline", "separate"])
@pytest.mark.parametrize("M", [512, 16], ids=["tcgen05", "few_rows"])
def test_noalloc_overflow_then_clean_inputs(cuda, redo, M):
    # The shared array still holds the first call's set flags when the second,
    # clean call of the same shape runs: every one of them must be rewritten,
    # or the second call would redo (and differ on) tiles it never flagged.
    # M = 16 takes the few-row kernel, which writes its flags per column tile.
    lib = _lib.load()
    g = torch.Generator().manual_seed(21 + M)
    N, K = 640, 384
    bad_a = torch.randn(M, K, generator=g)
    bad_b = torch.randn(K, N, generator=g)
    bad_a[torch.randperm(M, generator=g)[: max(1, M // 64)]] *= 256.0
    bad_b[:, torch.randperm(N, generator=g)[: N // 64]] *= 256.0
    bad = (bad_a.half().to(cuda), bad_b.half().to(cuda))
    clean = (torch.randn(M, K, generator=g).half().to(cuda), torch.randn(K, N, generator=g).half().to(cuda))
    mode = {"inline": _lib.REDO_INLINE, "separate": _lib.REDO_SEPARATE}[redo]
    prev = lib.f16acc_set_redo_mode(mode)
    try:
        assert _flagged_tiles(lib, *bad) > 0 and _flagged_tiles(lib, *clean) == 0
        for a, b in (bad, clean, bad, clean):
            ref = _reference(lib, a, b, torch.float32, True)
            rc, c = _noalloc(lib, a, b, torch.float32, True)
            assert rc == _lib.OK, _lib.strerror(rc)
            torch.cuda.synchronize()
            assert torch.equal(c, ref)
    finally:
        lib.f16acc_set_redo_mode(prev)


def test_noalloc_rejects_outputs_beyond_its_fixed_array(cuda):
    lib = _lib.load()
    # 65536 tiles of 128 x 128 fit; one more tile row does not.  Nothing is launched
    # for the rejected call, so tiny operand buffers suffice (only sizes are read).
    a = torch.zeros(8, 8, device=cuda, dtype=torch.float16)
    c = torch.zeros(8, 8, device=cuda, dtype=torch.float32)
    stream = torch.cuda.current_stream(cuda).cuda_stream
    M, N, K = 128 * 257, 128 * 256, 64  # 65792 tiles
    rc = lib.f16acc_gemm_noalloc(a.data_ptr(), K, 1, a.data_ptr(), N, 1, c.data_ptr(), N, 1, _lib.OUT_F32,
                                 M, N, K, 1, cuda.index or 0, stream)
    assert rc == _lib.ERR_TOO_LARGE
    assert b"F16ACC_NOALLOC_MAX_TILES" in lib.f16acc_strerror(rc)
