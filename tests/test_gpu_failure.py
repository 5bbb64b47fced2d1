"""Failure detection on the GPU without a fault: a bounded device wait is made
to run out on purpose (an mbarrier that nothing arrives on, a 1 ms limit), and
the kernel must end on its own, report the documented status code, stop the
CTA's other waiters through its abort flag, and leave the context usable for
the next product.  The product kernels use the same wait (mbar_wait) with a
4 s limit; their give-up path is what this exercises.  The named-barrier
release of the chunked kernel is checked on the CPU instead
(test_release_protocol.py)."""

import numpy as np
import pytest
import torch

import f16acc_b200 as f16acc
from f16acc_b200 import _lib
from f16acc_b200.kernel import device_status
from oracle import oracle as O
from tests.helpers import chunk_ulp_bound

pytestmark = pytest.mark.gpu

STATUS_TIMEOUT_PROBE = 0x104


def test_expired_wait_reports_status_and_the_context_stays_usable(cuda):
    lib = _lib.load()
    assert device_status(0, reset=True) == 0
    out = torch.full((3,), -1, dtype=torch.int64, device=cuda)
    stream = torch.cuda.current_stream(cuda).cuda_stream
    limit_ns = 1_000_000
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    assert lib.f16acc_selftest_wait_timeout(limit_ns, out.data_ptr(), 0, stream) == _lib.OK
    e1.record()
    torch.cuda.synchronize()
    waited_ns, left, wrongly_ok = out.cpu().tolist()
    assert wrongly_ok == 0
    assert limit_ns <= waited_ns < 200 * limit_ns  # gave up after its own limit, not the products' 4 s
    assert left == 64  # every other waiter left on the abort flag
    assert e0.elapsed_time(e1) < 1000.0  # ms: the kernel ended long before any 4 s limit
    assert device_status(0, reset=False) == STATUS_TIMEOUT_PROBE  # stays set until reset
    assert device_status(0, reset=True) == STATUS_TIMEOUT_PROBE
    assert device_status(0, reset=True) == 0
    # the next product runs normally and reports nothing
    g = torch.Generator().manual_seed(9)
    a = torch.randn(384, 320, generator=g).half()
    b = torch.randn(320, 256, generator=g).half()
    c = f16acc.mm(a.to(cuda), b.to(cuda), torch.float32).cpu().numpy()
    ref, _ = O.gemm_chunked(a.numpy(), b.numpy(), round_every=16)
    assert (np.abs(c - ref) <= chunk_ulp_bound(a.numpy(), b.numpy())).all()
    assert device_status(0, reset=True) == 0


def test_selftest_rejects_limits_outside_the_product_bound(cuda):
    lib = _lib.load()
    out = torch.zeros(3, dtype=torch.int64, device=cuda)
    stream = torch.cuda.current_stream(cuda).cuda_stream
    assert lib.f16acc_selftest_wait_timeout(0, out.data_ptr(), 0, stream) == _lib.ERR_INVALID_ARGUMENT
    assert lib.f16acc_selftest_wait_timeout(5_000_000_000, out.data_ptr(), 0, stream) == _lib.ERR_INVALID_ARGUMENT
    assert lib.f16acc_selftest_wait_timeout(1000, None, 0, stream) == _lib.ERR_INVALID_ARGUMENT
