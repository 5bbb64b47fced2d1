"""The raw-rate probes (counterparts of the reference's bench/rate.py and
bench/chunkrate.py) run, end without a device status, and report rates in a
plausible range: the tcgen05 MMA-only probes near the dense peak with either
accumulator, the chunk pipeline and the mma.sync chunkrate analogue well
above zero.  The measured table is in profiles/chunk_rate_probes.md."""

import math

import pytest
import torch

from f16acc_b200 import probe_rate
from f16acc_b200.kernel import device_status

pytestmark = pytest.mark.gpu


def test_probes_run_and_report_rates(cuda):
    rates = {}
    for mode, name, epi, unit in probe_rate.PROBES:
        sms, ms, tflops, _ = probe_rate.run(mode, epi, 2048, 2, cuda, unit)
        assert sms > 0 and ms > 0 and math.isfinite(tflops), name
        rates[(mode, epi)] = tflops
    assert device_status(0, reset=True) == 0
    # FP16 and FP32 accumulators run at the same tensor rate on B200
    assert 0.8 < rates[(0, 2)] / rates[(1, 2)] < 1.25
    assert rates[(0, 2)] > 1000.0
    assert 100.0 < rates[(2, 2)] < rates[(0, 2)]
    assert rates[(32, 0)] > 100.0
