"""Failure detection on the GPU without a fault: a bounded wait that runs out ends in a status word
the host reads, and the device stays usable.

mas_selftest_bounded_wait launches one thread that waits on an mbarrier nothing completes (a flag
that nothing sets), with a short limit, through the same bounded wait every bulk-copy consumer in
the library uses; on expiry it sets MAS_STATUS_COPY_TIMEOUT in the library fault word. No trap, no
assert, no out-of-bounds access: the context is intact afterwards, which the test checks by running
an op and comparing it with the oracle.
"""
from __future__ import annotations

import time

import pytest
import torch

import mas_b200
import oracle
from mas_b200 import _lib
from parity import assert_ulp

pytestmark = pytest.mark.gpu


def test_wait_that_runs_out_reports_a_timeout_and_the_device_stays_usable(cuda):
    mas_b200.read_fault_word(cuda.index, clear=True)
    stream = torch.cuda.current_stream().cuda_stream
    t0 = time.perf_counter()
    assert _lib.lib.mas_selftest_bounded_wait(20_000_000, stream) == 0  # 20 ms
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert waited >= 0.015, waited  # the wait ran to its limit ...
    assert waited < 1.5, waited     # ... and no further
    assert mas_b200.read_fault_word(cuda.index, clear=True) & _lib.STATUS_COPY_TIMEOUT
    assert mas_b200.read_fault_word(cuda.index) == 0  # cleared

    # the context is still good: an op runs and matches the oracle
    g = torch.Generator().manual_seed(3)
    x = torch.randn(5, 2 * 256, generator=g).to(torch.bfloat16)
    assert_ulp(mas_b200.silu_and_mul(x.to(cuda)).cpu(), oracle.silu_and_mul(x), what="after the timeout")
    assert mas_b200.read_fault_word(cuda.index) == 0


def test_selftest_limits_are_checked(cuda):
    assert _lib.lib.mas_selftest_bounded_wait(0, None) == _lib.ERR_INVALID_ARGUMENT
    assert _lib.lib.mas_selftest_bounded_wait(3_000_000_000, None) == _lib.ERR_INVALID_ARGUMENT
