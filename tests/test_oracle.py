"""The CPU oracle pinned against the reference itself.

tests/golden/reference_cases.npz holds inputs and outputs of the reference's
own Triton kernels (steppergg/f16acc f16acc/kernel.py:63-81), run under
Triton's CPU interpreter by tests/golden/make_golden.py.  The oracle must
reproduce them: tile flags exactly, the overflow known answer exactly
(tests/test_f16acc.py:91-101), and every other value to within one FP16
rounding of each chunk sum (the reference sums a chunk in FP32 in numpy's
order, the oracle exactly, before the FP16 rounding)."""

import os

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import chunk_ulp_bound, rel

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "reference_cases.npz")


def _cases():
    z = np.load(GOLDEN)
    names = sorted({k.split("/")[0] for k in z.files})
    out = []
    for n in names:
        d = {k.split("/", 1)[1]: z[k] for k in z.files if k.startswith(n + "/")}
        out.append((n, d))
    return out


CASES = _cases()


def _b(d):
    return d["b"] if "b" in d else d["b_t"].T  # b_t stored contiguous: b is its transposed view


@pytest.mark.parametrize("name,d", CASES, ids=[c[0] for c in CASES])
def test_oracle_matches_reference_kernel(name, d):
    a, b = d["a"], _b(d)
    ref = d["c"].astype(np.float64)
    chunked = bool(d["chunked"])
    if chunked:
        c, flags = O.gemm_chunked(a, b, tile=(64, 64), redo=True)
        assert (flags.reshape(-1) == d["flags"].astype(np.uint8)).all(), "tile flags differ from the reference"
    else:
        c = O.gemm_f32acc(a, b)
    if str(d["out"]) == "torch.float16":
        c = O.round_f16(c)
    c = c.astype(np.float64)
    if "overflow_kat" in name:
        assert (c == 100.0).all() and (ref == 100.0).all()
        return
    if chunked:
        bound = chunk_ulp_bound(a, b, ulps=1.0)
        if str(d["out"]) == "torch.float16":
            bound = bound + 2 * np.maximum(np.abs(ref) * 2.0 ** -11, 2.0 ** -25)
        flagged = np.repeat(np.repeat(d["flags"].reshape((a.shape[0] + 63) // 64, -1), 64, 0), 64, 1)
        flagged = flagged[: a.shape[0], : b.shape[1]].astype(bool)
        bound = np.where(flagged, np.abs(ref) * 2.0 ** -22 + 1e-30, bound)
        assert (np.abs(c - ref) <= bound).all(), float(np.abs(c - ref).max())
    else:
        assert np.abs(c - ref).max() <= np.abs(ref).max() * 2.0 ** -20


def test_golden_overflow_case_is_flagged_and_repaired():
    d = dict(CASES)["overflow_kat_64x64x64"]
    assert d["flags"].tolist() == [1]
    assert (d["c"].astype(np.float64) == 100.0).all()


def test_overflow_known_answer_exact():
    # tests/test_f16acc.py:91-101 at its own size: each 32-long chunk sums to
    # +-96000 (inf in FP16); the FP32 redo gives exactly 100
    x = np.full((256, 64), 100.0, dtype=np.float16)
    w = np.empty((128, 64), dtype=np.float16)
    w[:, :32] = 30.0
    w[:, 32:] = -30.0
    w[:, 63] = -29.0
    c, flags = O.gemm_chunked(x, w.T, tile=(128, 128), redo=False)
    assert np.isnan(c).all() and flags.all()
    c, flags = O.gemm_chunked(x, w.T, tile=(128, 128), redo=True)
    assert (c == 100.0).all()


@pytest.mark.parametrize("round_every", [16, 32])
def test_config1_accuracy(round_every):
    # 512^3, U[-1,1] (seeded), within 1e-3 of FP64
    rng = np.random.default_rng(0)
    a = rng.uniform(-1, 1, (512, 512)).astype(np.float16)
    b = rng.uniform(-1, 1, (512, 512)).astype(np.float16)
    ref = O.gemm_f64(a, b)
    c, _ = O.gemm_chunked(a, b, round_every=round_every)
    assert rel(c, ref) < 1e-3
    assert rel(O.gemm_f32acc(a, b), ref) < 1e-6


def test_chunks_start_at_absolute_offsets():
    # a chunk is K[32c, 32c+32): moving mass across a chunk boundary changes
    # which values are rounded together
    a = np.zeros((1, 64), dtype=np.float16)
    b = np.zeros((64, 1), dtype=np.float16)
    a[0, 31] = a[0, 32] = 1.0
    b[31, 0] = 2048.0
    b[32, 0] = 1.0
    c, _ = O.gemm_chunked(a, b)
    # chunk 0 = 2048, chunk 1 = 1: both exact, sum 2049 exact in FP32
    assert c[0, 0] == 2049.0
    # within one chunk 2048 + 1 rounds to 2048 in FP16 (ulp 2 at 2048)
    a2 = np.zeros((1, 64), dtype=np.float16)
    a2[0, 30] = a2[0, 31] = 1.0
    b2 = np.zeros((64, 1), dtype=np.float16)
    b2[30, 0] = 2048.0
    b2[31, 0] = 1.0
    c2, _ = O.gemm_chunked(a2, b2)
    assert c2[0, 0] == 2048.0


def test_strided_views_match_contiguous():
    rng = np.random.default_rng(3)
    a = rng.standard_normal((70, 90)).astype(np.float16)
    w = rng.standard_normal((50, 90)).astype(np.float16)
    c1, _ = O.gemm_chunked(a, w.T)
    c2, _ = O.gemm_chunked(a, np.ascontiguousarray(w.T))
    assert np.array_equal(c1, c2)
    big = rng.standard_normal((140, 200)).astype(np.float16)
    c3, _ = O.gemm_chunked(big[::2, :90], np.ascontiguousarray(w.T))
    c4, _ = O.gemm_chunked(np.ascontiguousarray(big[::2, :90]), np.ascontiguousarray(w.T))
    assert np.array_equal(c3, c4)


def test_empty_k_gives_zeros_and_rel_keeps_nan():
    a = np.zeros((4, 0), dtype=np.float16)
    b = np.zeros((0, 3), dtype=np.float16)
    c, _ = O.gemm_chunked(a, b)
    assert (c == 0).all()
    x = np.array([[1.0, np.nan]], dtype=np.float32)
    assert np.isnan(O.rel(x, np.ones((1, 2))))
