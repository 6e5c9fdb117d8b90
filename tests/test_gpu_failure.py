"""Failure detection without a GPU fault: the pipelines' bounded wait, run on
an mbarrier that nothing completes, gives up after its limit, reports through
the fault word (uk_cuda_pipeline_fault, bit 16) and leaves the context usable;
the positive control completes normally."""
import time

import numpy as np
import pytest

import unikern_b200.abi as abi
from oracle import oracle as O
from uk_testutil import dev, empty, host

pytestmark = pytest.mark.gpu


def run_selftest(arrive, timeout_ns):
    import torch
    status = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    abi.check(abi.lib().uk_cuda_selftest_wait(arrive, timeout_ns, status.data_ptr(), None))
    torch.cuda.synchronize()
    return int(status.item())


def test_bounded_wait_expires_and_reports():
    assert abi.lib().uk_cuda_pipeline_fault() == 0
    t0 = time.perf_counter()
    assert run_selftest(0, 2_000_000) == 0        # 2 ms limit, nothing arrives
    assert time.perf_counter() - t0 < 5.0
    assert abi.lib().uk_cuda_pipeline_fault() == 16
    assert abi.lib().uk_cuda_pipeline_fault() == 0   # read-and-clear
    # the context is usable: a GEMM right after is exact on the sawtooth instance
    A = O.sawtooth("A", 256 * 256).reshape(256, 256)
    B = O.sawtooth("B", 256 * 256).reshape(256, 256)
    Cm = empty((256, 256))
    abi.gemm_f32(dev(A), dev(B), Cm)
    assert np.array_equal(host(Cm), O.gemm_f32(A, B, threads=8))
    assert abi.lib().uk_cuda_pipeline_fault() == 0


def test_bounded_wait_completes_when_the_barrier_does():
    assert run_selftest(1, 2_000_000) == 1
    assert abi.lib().uk_cuda_pipeline_fault() == 0


def test_selftest_limits_are_checked():
    import torch
    status = torch.zeros((1,), dtype=torch.int32, device="cuda")
    for bad in (0, 999, 2_000_000_000):
        assert abi.lib().uk_cuda_selftest_wait(0, bad, status.data_ptr(), None) == 2
