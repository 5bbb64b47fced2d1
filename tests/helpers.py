"""Shared test helpers: the reference's rel() metric and the per-element bound
on how far two correct chunked results may differ."""

import numpy as np


def rel(x, ref):
    """max|x - ref| / max|ref| (steppergg/f16acc tests/test_f16acc.py:11-12)."""
    x = np.asarray(x, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.abs(x - ref).max() / np.abs(ref).max())


def ulp16(x):
    """Spacing of FP16 numbers at |x| (subnormal spacing below 2^-14)."""
    ax = np.abs(np.asarray(x, dtype=np.float64))
    e = np.floor(np.log2(np.maximum(ax, 2.0 ** -14)))
    return 2.0 ** (e - 10)


def chunk_ulp_bound(a16, b16, ulps=2.0, chunk=32):
    """Per-element bound on |x - y| for two chunked products that may round
    each FP16 chunk sum differently (where and how often the FP16 accumulator
    rounds inside a chunk is hardware defined): `ulps` FP16 ulps at the
    magnitude of the chunk's absolute sum (an upper bound on every partial sum
    inside the chunk, so cancellation is covered), plus FP32 rounding of the
    running sums."""
    a = np.asarray(a16, dtype=np.float64)
    b = np.asarray(b16, dtype=np.float64)
    K = a.shape[1]
    bound = np.zeros((a.shape[0], b.shape[1]))
    run = np.zeros_like(bound)
    aa, ab = np.abs(a), np.abs(b)
    for k0 in range(0, K, chunk):
        absum = aa[:, k0:k0 + chunk] @ ab[k0:k0 + chunk]
        run += absum
        bound += ulps * ulp16(absum)
    nch = max(1, (K + chunk - 1) // chunk)
    return bound + nch * run * 2.0 ** -23 + 1e-30


def chunk_ulp_bound_torch(a16, b16, ulps=2.0, chunk=32):
    """chunk_ulp_bound computed on the operands' device in float64 (torch
    tensors [M, K] and [K, N], any strides): the same bound for products too
    large for a numpy loop over the chunks."""
    import torch

    a = a16.double().abs()
    b = b16.double().abs()
    K = a.shape[1]
    bound = torch.zeros(a.shape[0], b.shape[1], dtype=torch.float64, device=a.device)
    run = torch.zeros_like(bound)
    for k0 in range(0, K, chunk):
        absum = a[:, k0:k0 + chunk] @ b[k0:k0 + chunk]
        run += absum
        e = torch.floor(torch.log2(torch.clamp(absum, min=2.0 ** -14)))
        bound += ulps * torch.exp2(e - 10)
    nch = max(1, (K + chunk - 1) // chunk)
    return bound + nch * run * 2.0 ** -23 + 1e-30
