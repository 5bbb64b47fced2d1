"""Chunked FP16-accumulate GEMM on B200: C = A @ B, fp16 in, FP32 sum of
FP16-accumulated 32-long K chunks.

Host-side mirror of steppergg/f16acc f16acc/kernel.py:84-105 (`mm`): the same
signature, the same ValueError checks and messages, C allocated here with
`out_dtype`, a per-call flag workspace from the caching allocator, and an
asynchronous launch on the current stream with no host sync.  The work itself
is the native library (include/f16acc.h): a warp-specialised tcgen05/TMA
kernel when the operands allow TMA, a few-row kernel for M <= 64 (M <= 32
when N > 32768), else a
warp-level mma.sync kernel that takes any strides.  Tiles whose FP16 chunk
overflowed are redone with FP32 accumulation on the device: inside the same
tcgen05 launch by default, otherwise by a second kernel launched behind the
first on the stream.

Unlike the reference there is no autotuner state: the kernel choice is a pure
function of the operands, so `mm` may be called from several threads.
"""

from __future__ import annotations

import functools

import torch

from . import _lib

_OUT_CODES = {torch.float16: _lib.OUT_F16, torch.float32: _lib.OUT_F32, torch.bfloat16: _lib.OUT_BF16}

# The current stream's raw handle for a device index: torch's own accessor
# (the one its generated kernels launch through) when present, which costs a
# fraction of building a torch.cuda.Stream object per call.
if hasattr(torch._C, "_cuda_getCurrentRawStream"):
    _raw_stream = torch._C._cuda_getCurrentRawStream
else:  # pragma: no cover - older torch
    def _raw_stream(index):
        return torch.cuda.current_stream(index).cuda_stream


def _device_index(t) -> int:
    index = t.device.index
    return index if index is not None else torch.cuda.current_device()


def _check(a, b):
    # real checks, not asserts (kernel.py:85-90): a bad shape or dtype would
    # make the kernel read past the end of b
    if a.dim() != 2 or b.dim() != 2 or a.shape[1] != b.shape[0]:
        raise ValueError(f"mm needs (M, K) @ (K, N), got {tuple(a.shape)} @ {tuple(b.shape)}")
    if a.dtype != torch.float16 or b.dtype != torch.float16 or not (a.is_cuda and b.is_cuda) or a.device != b.device:
        raise ValueError("mm needs fp16 CUDA tensors on the same device")


def _raise(rc: int):
    msg = _lib.strerror(rc)
    if rc in (_lib.ERR_INVALID_ARGUMENT, _lib.ERR_UNSUPPORTED):
        raise ValueError(msg)
    raise RuntimeError(f"f16acc_b200: {msg} (code {rc})")


@functools.lru_cache(maxsize=4096)
def workspace_bytes(M: int, N: int, K: int) -> int:
    return int(_lib.load().f16acc_workspace_bytes(M, N, K))


def _check_bias(bias, a, n):
    if not (isinstance(bias, torch.Tensor) and bias.dtype == torch.float16 and bias.device == a.device):
        raise ValueError("bias must be an fp16 tensor on the operands' device")
    if bias.dim() != 1 or bias.shape[0] != n:
        raise ValueError(f"bias must have shape ({n},), got {tuple(bias.shape)}")


def mm_ex(a, b, out_dtype=torch.float16, chunked=True, *, variant=_lib.VARIANT_AUTO, out=None, workspace=None,
          bias=None):
    """`mm` with the kernel variant forced, optional caller-owned output and
    workspace (tests and benchmarks read the per-tile flags from it), and an
    optional fp16 bias[N] added in the epilogue (see `mm_bias`).
    Returns (c, workspace)."""
    _check(a, b)
    if bias is not None:
        _check_bias(bias, a, b.shape[1])
    code = _OUT_CODES.get(out_dtype)
    if code is None:
        raise ValueError(f"mm supports out_dtype float16, float32 or bfloat16, got {out_dtype}")
    lib = _lib.load()
    M, K = a.shape
    N = b.shape[1]
    if out is None:
        out = torch.empty(M, N, device=a.device, dtype=out_dtype)
    elif out.shape != (M, N) or out.dtype != out_dtype or out.device != a.device:
        raise ValueError("out must be an (M, N) tensor of out_dtype on the operands' device")
    ws_ptr, ws_len = None, 0
    if chunked:
        if workspace is None:
            workspace = torch.empty(workspace_bytes(M, N, K), dtype=torch.uint8, device=a.device)
        else:
            # the flags must fit; the tail split runs only in a workspace_bytes() workspace
            need = -(-M // 128) * -(-N // 128) * 16
            if workspace.numel() < need or workspace.device != a.device or workspace.dtype != torch.uint8:
                raise ValueError(f"workspace must be a uint8 tensor of at least {need} bytes on the operands' device")
        ws_ptr, ws_len = workspace.data_ptr(), workspace.numel()
    dev = _device_index(a)
    stream = _raw_stream(dev)
    if bias is None:
        rc = lib.f16acc_gemm_ex(a.data_ptr(), a.stride(0), a.stride(1), b.data_ptr(), b.stride(0), b.stride(1),
                                out.data_ptr(), out.stride(0), out.stride(1), code, M, N, K, 1 if chunked else 0,
                                ws_ptr, ws_len, dev, stream, int(variant))
    else:
        rc = lib.f16acc_gemm_bias(a.data_ptr(), a.stride(0), a.stride(1), b.data_ptr(), b.stride(0), b.stride(1),
                                  bias.data_ptr(), bias.stride(0), out.data_ptr(), out.stride(0), out.stride(1),
                                  code, M, N, K, 1 if chunked else 0, ws_ptr, ws_len, dev, stream, int(variant))
    if rc != _lib.OK:
        _raise(rc)
    return out, workspace


def mm_bias(a, b, bias, out_dtype=torch.float16, chunked=True):
    """C = a @ b + bias with the bias added in the GEMM's epilogue.

    Bit-identical to the reference's `y = mm(a, b); y += bias`
    (patch.py:28-30) for an fp16 `bias` of shape (N,): the product is rounded
    to out_dtype, the bias added in FP32 and the sum rounded once more, without
    the second pass over y."""
    return mm_ex(a, b, out_dtype, chunked, bias=bias)[0]


def mm(a, b, out_dtype=torch.float16, chunked=True):
    """C = a @ b for fp16 CUDA matrices of any strides (kernel.py:84).

    chunked=True: each 32-long K chunk is accumulated in FP16 and the chunks
    are summed in FP32; tiles where a chunk overflowed FP16 are redone with
    FP32 accumulation on the device.  chunked=False: plain FP32 accumulation.
    """
    _check(a, b)
    code = _OUT_CODES.get(out_dtype)
    if code is None:
        raise ValueError(f"mm supports out_dtype float16, float32 or bfloat16, got {out_dtype}")
    lib = _lib.load()
    M, K = a.shape
    N = b.shape[1]
    c = torch.empty(M, N, device=a.device, dtype=out_dtype)
    ws_ptr, ws_len, ws = None, 0, None
    if chunked:
        ws = torch.empty(workspace_bytes(M, N, K), dtype=torch.uint8, device=a.device)
        ws_ptr, ws_len = ws.data_ptr(), ws.numel()
    dev = _device_index(a)
    rc = lib.f16acc_gemm(a.data_ptr(), a.stride(0), a.stride(1), b.data_ptr(), b.stride(0), b.stride(1),
                         c.data_ptr(), c.stride(0), c.stride(1), code, M, N, K, 1 if chunked else 0,
                         ws_ptr, ws_len, dev, _raw_stream(dev))
    if rc != _lib.OK:
        _raise(rc)
    return c


def mm_phase(phase, a, b, out, workspace, chunked=True, variant=_lib.VARIANT_AUTO):
    """Issue one of the two launches of a chunked product into caller-owned
    `out` and `workspace`: phase "main" (C and tile flags) or "redo" (FP32
    recompute of flagged tiles).  main then redo on one stream == mm_ex."""
    _check(a, b)
    code = _OUT_CODES.get(out.dtype)
    if code is None:
        raise ValueError(f"unsupported output dtype {out.dtype}")
    lib = _lib.load()
    fn = {"main": lib.f16acc_gemm_main, "redo": lib.f16acc_gemm_redo}[phase]
    M, K = a.shape
    N = b.shape[1]
    dev = _device_index(a)
    ws_ptr, ws_len = (workspace.data_ptr(), workspace.numel()) if workspace is not None else (None, 0)
    rc = fn(a.data_ptr(), a.stride(0), a.stride(1), b.data_ptr(), b.stride(0), b.stride(1),
            out.data_ptr(), out.stride(0), out.stride(1), code, M, N, K, 1 if chunked else 0,
            ws_ptr, ws_len, dev, _raw_stream(dev), int(variant))
    if rc != _lib.OK:
        _raise(rc)


def plan(a, b, variant=_lib.VARIANT_AUTO):
    """The kernel and tile grid `mm_ex` would use for these operands."""
    _check(a, b)
    p = _lib.Plan()
    rc = _lib.load().f16acc_get_plan(a.data_ptr(), a.stride(0), a.stride(1), b.data_ptr(), b.stride(0), b.stride(1),
                                     a.shape[0], b.shape[1], a.shape[1], int(variant), p)
    if rc != _lib.OK:
        _raise(rc)
    return {"variant": p.variant, "tile": (p.tile_m, p.tile_n), "tiles": (p.tiles_m, p.tiles_n)}


def tile_flags(workspace, plan_):
    """Per-tile overflow flags from a chunked call's workspace: a bool tensor
    [tiles_m, tiles_n] on the workspace's device."""
    tm, tn = plan_["tiles"]
    fb = int(_lib.load().f16acc_flag_bytes_per_tile())
    return workspace[: tm * tn * fb].view(tm * tn, fb).ne(0).any(dim=1).view(tm, tn)


def device_status(device: int = 0, reset: bool = True) -> int:
    """Synchronise `device` and return the kernels' status word (0 = no wait
    timed out), clearing it when `reset`."""
    return int(_lib.load().f16acc_device_status(device, 1 if reset else 0))
