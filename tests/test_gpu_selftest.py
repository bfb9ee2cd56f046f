"""The kernels' bounded waits, exercised on the GPU without a fault: a wait on
an mbarrier that nothing completes gives up after its budget, reports
STATUS_TIMEOUT in the status word, and leaves the CUDA context usable."""

from __future__ import annotations

import time

import pytest
import torch

from asrback_b200 import _native

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_reports_timeout():
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    start = time.perf_counter()
    _native.call("asrback_selftest_bounded_wait", 20_000_000, status.data_ptr(), stream)
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - start
    assert status.item() & _native.STATUS_TIMEOUT
    assert 0.015 < elapsed < 5.0, elapsed
    # The context still runs work.
    x = torch.arange(1000, device="cuda", dtype=torch.float32)
    assert x.sum().item() == 499500.0
