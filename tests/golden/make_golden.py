"""Generate the golden fixtures in tests/golden/reference_cases.npz.

Runs the REFERENCE implementation itself -- the Triton kernels `_gemm` and
`_redo` of steppergg/f16acc (f16acc/kernel.py:63-81) -- under Triton's CPU
interpreter (TRITON_INTERPRET=1), on small seeded inputs, and stores inputs,
outputs and tile flags.  The reference cannot run on the GPU box (it is not
shipped there), so the fixtures carry its behaviour to the tests.

Run in the build container only, where the reference is mounted:
    python tests/golden/make_golden.py /path/to/reference
The reference's host wrapper `mm()` (kernel.py:84-105) rejects CPU tensors, so
the jitted kernels are launched directly with the same argument list `mm()`
builds (kernel.py:96-104), with one fixed tile config (BM=BN=64, BK=32, G=8;
one of the shapes `CONFIGS` allows, kernel.py:16-19).
"""

import os
import sys

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

BM = BN = 64


def run_reference(K_mod, a, b, out_dtype, chunked):
    M, K = a.shape
    N = b.shape[1]
    c = torch.empty(M, N, dtype=out_dtype)
    tiles = ((M + BM - 1) // BM) * ((N + BN - 1) // BN)
    flags = torch.zeros(tiles, dtype=torch.int8)
    args = (a, b, c, flags, M, N, K, a.stride(0), a.stride(1), b.stride(0), b.stride(1), c.stride(0), c.stride(1))
    K_mod._gemm.fn[(tiles,)](*args, CHUNKED=chunked, I64=False, BM=BM, BN=BN, BK=32, G=8)
    flags_main = flags.clone()
    if chunked:
        K_mod._redo[(tiles,)](*args, I64=False, BM=BM, BN=BN, BK=32, G=8)
    return c, flags_main


def main(ref_root):
    sys.path.insert(0, ref_root)
    from f16acc import kernel as K_mod

    cases = {}

    def add(name, a, b, out_dtype=torch.float32, chunked=True):
        c, flags = run_reference(K_mod, a, b, out_dtype, chunked)
        cases[name] = dict(a=a.contiguous().numpy(), b=b.numpy().copy() if b.is_contiguous() else None,
                           b_t=None if b.is_contiguous() else b.t().contiguous().numpy(),
                           c=c.numpy(), flags=flags.numpy(), chunked=np.array(chunked),
                           out=np.array(str(out_dtype)))

    g = torch.Generator().manual_seed(0)
    # config-1 style: U[-1,1], fp32 out (BASELINE config 1 distribution, shrunk)
    a = (torch.rand(64, 96, generator=g) * 2 - 1).half()
    b = (torch.rand(96, 64, generator=g) * 2 - 1).half()
    add("uniform_64x96x64", a, b)
    # ragged: K tail not a multiple of 32, M and N not multiples of the tile
    a = torch.randn(50, 77, generator=g).half()
    b = torch.randn(77, 70, generator=g).half()
    add("ragged_50x77x70", a, b)
    # config-2 distribution N(0,1)/sqrt(K)*4, fp16 out
    a = (torch.randn(96, 160, generator=g) / 160 ** 0.5 * 4).half()
    b = (torch.randn(160, 96, generator=g) / 160 ** 0.5 * 4).half()
    add("scaled_96x160x96_f16out", a, b, out_dtype=torch.float16)
    # nn.Linear weight layout: b = w.t() (strides (1, K))
    a = torch.randn(64, 128, generator=g).half()
    w = torch.randn(80, 128, generator=g).half()
    add("wt_64x128x80", a, w.t())
    # chunked=False: plain FP32 accumulation
    a = torch.randn(64, 64, generator=g).half()
    b = torch.randn(64, 64, generator=g).half()
    add("fp32acc_64x64x64", a, b, chunked=False)
    # known answer (tests/test_f16acc.py:91-101): chunk sums +-96000 overflow fp16,
    # the redo must give exactly 100 everywhere
    x = torch.full((64, 64), 100.0).half()
    w = torch.empty(64, 64).half()
    w[:, :32] = 30.0
    w[:, 32:] = -30.0
    w[:, 63] = -29.0
    add("overflow_kat_64x64x64", x, w.t(), out_dtype=torch.float16)
    # overflow stress in the style of BASELINE config 4, shrunk: scaled rows/cols
    a = torch.randn(128, 128, generator=g).half()
    b = torch.randn(128, 128, generator=g).half()
    a[5] *= 64
    b[:, 77] *= 64
    add("overflow_stress_128x128x128", a, b)

    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_cases.npz")
    flat = {}
    for name, d in cases.items():
        for k, v in d.items():
            if v is not None:
                flat[f"{name}/{k}"] = v
    np.savez_compressed(out, **flat)
    print("wrote", out, "cases:", list(cases))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path to the steppergg/f16acc checkout>")
    main(sys.argv[1])
