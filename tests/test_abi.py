"""The C-ABI library loads and exports every symbol include/f16acc.h declares;
host-only entry points answer without a GPU."""

import os
import re

import pytest

from f16acc_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "f16acc.h")


def _declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(f16acc_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_gemm_boundary():
    names = _declared()
    for n in ("f16acc_gemm", "f16acc_workspace_bytes", "f16acc_strerror"):
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for n in _declared():
        assert hasattr(lib, n), n
    assert set(_declared()) == set(_lib.SIGNATURES)


def test_workspace_and_messages():
    lib = _lib.load()
    fb = lib.f16acc_flag_bytes_per_tile()
    assert fb == 16
    # K too short for a tail split to pay (it must take 20 or more 64-wide
    # stages off a tile): the flags alone
    assert lib.f16acc_workspace_bytes(1, 1, 1) == fb
    assert lib.f16acc_workspace_bytes(129, 257, 7) == 2 * 3 * fb
    assert lib.f16acc_workspace_bytes(4096, 4096, 1600) == 32 * 32 * fb
    # otherwise the flags, 256-byte aligned, then 148 split counters and 512
    # bytes, then at most 148 partial tiles (4 per tile) of 128 x 128 FP32
    part = 128 * 128 * 4
    assert lib.f16acc_workspace_bytes(4096, 4096, 4096) == 32 * 32 * fb + 148 * 4 + 512 + 148 * part
    assert lib.f16acc_workspace_bytes(256, 128, 1664) == 256 + 148 * 4 + 512 + 2 * 4 * part
    for code in range(6):
        assert lib.f16acc_strerror(code)
    assert b"unknown" in lib.f16acc_strerror(99)
    assert b"sm_100a" in lib.f16acc_version()


def test_invalid_arguments_rejected_before_any_cuda_call():
    lib = _lib.load()
    # negative sizes and unknown output codes fail with INVALID_ARGUMENT, no device touched
    assert lib.f16acc_gemm(None, 0, 0, None, 0, 0, None, 0, 0, 0, -1, 1, 1, 1, None, 0, 0, None) == _lib.ERR_INVALID_ARGUMENT
    assert lib.f16acc_gemm(None, 0, 0, None, 0, 0, None, 0, 0, 7, 1, 1, 1, 1, None, 0, 0, None) == _lib.ERR_INVALID_ARGUMENT
    # empty products are a no-op
    assert lib.f16acc_gemm(None, 0, 0, None, 0, 0, None, 0, 0, 0, 0, 5, 5, 1, None, 0, 0, None) == _lib.OK
    assert lib.f16acc_gemm(None, 0, 0, None, 0, 0, None, 0, 0, 0, 5, 0, 5, 1, None, 0, 0, None) == _lib.OK


def test_device_ordinals_that_are_not_devices_are_invalid_arguments():
    # ordinal 63 is below the library's table size but no device of this
    # process (none at all on a CPU-only host)
    lib = _lib.load()
    assert lib.f16acc_gemm(None, 0, 0, None, 0, 0, None, 0, 0, 0, 5, 5, 5, 1, None, 0, 63, None) == \
        _lib.ERR_INVALID_ARGUMENT
    assert lib.f16acc_gemm_noalloc(None, 0, 0, None, 0, 0, None, 0, 0, 0, 5, 5, 5, 1, 63, None) == \
        _lib.ERR_INVALID_ARGUMENT
    assert lib.f16acc_gemm_noalloc(None, 0, 0, None, 0, 0, None, 0, 0, 0, 5, 5, 5, 1, -1, None) == \
        _lib.ERR_INVALID_ARGUMENT
    assert lib.f16acc_device_status(63, 0) == -1


def test_plan_without_a_gpu_is_mma_sync_or_tcgen05():
    p = _lib.Plan()
    rc = _lib.load().f16acc_get_plan(16, 64, 1, 16, 1, 64, 128, 128, 64, _lib.VARIANT_MMA_SYNC, p)
    assert rc == _lib.OK and p.variant == _lib.VARIANT_MMA_SYNC and (p.tile_m, p.tile_n) == (128, 128)
    assert (p.tiles_m, p.tiles_n) == (1, 1)


def test_tuning_knobs_validate_and_return_the_previous_setting():
    lib = _lib.load()
    assert lib.f16acc_set_fp32_tiles(7) == _lib.ERR_INVALID_ARGUMENT
    assert lib.f16acc_set_tail_split(2) == _lib.ERR_INVALID_ARGUMENT
    assert lib.f16acc_set_tail_split(_lib.TAIL_SPLIT_OFF) == _lib.TAIL_SPLIT_ON
    assert lib.f16acc_set_tail_split(_lib.TAIL_SPLIT_ON) == _lib.TAIL_SPLIT_OFF
    assert lib.f16acc_set_fp32_tiles(_lib.FP32_TILES_WIDE) == _lib.FP32_TILES_AUTO
    assert lib.f16acc_set_fp32_tiles(_lib.FP32_TILES_AUTO) == _lib.FP32_TILES_WIDE
    assert lib.f16acc_set_schedule(5) == _lib.ERR_INVALID_ARGUMENT
    assert lib.f16acc_set_redo_mode(5) == _lib.ERR_INVALID_ARGUMENT


def test_workspace_bytes_holds_every_tail_split_plan():
    """Whatever SM count the split plans for (all 148 SMs or a cap), the
    workspace f16acc_workspace_bytes reports holds the flags, the counters and
    the partial tiles of that plan, so a caller sizing by it never loses the
    split.  The plan restated: tiles past the last full wave, S = min(4,
    SMs / those tiles, stages / 6) parts, used when it takes 20 or more
    64-wide stages off a tile."""
    lib = _lib.load()
    part = 128 * 128 * 4
    for M in (128, 300, 2048, 8192):
        for N in (128, 256, 1536, 8960):
            for K in (1024, 1600, 1664, 4096, 8960):
                tiles = -(-M // 128) * -(-N // 128)
                nkb = -(-K // 64)
                flags = tiles * 16
                for sms in (148, 132, 100, 64):
                    r = tiles if tiles < sms else tiles % sms
                    if r == 0:
                        continue
                    s = min(4, sms // r, nkb // 6)
                    if s < 2 or s * r > 148 or nkb - nkb // s < 20:
                        continue
                    need = -(-flags // 256) * 256 + 148 * 4 + 512 + s * r * part
                    assert lib.f16acc_workspace_bytes(M, N, K) >= need, (M, N, K, sms)
