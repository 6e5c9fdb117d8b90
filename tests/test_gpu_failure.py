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


# ---- the device-side barrier of the ranks (uk_cuda_peer_barrier) ---------------------
# On one GPU, with a second local array standing in for rank 1's: rank 1's post
# never comes unless the test writes it, so the bounded wait runs out.

def _peer_barrier(own, other, epoch, timeout_ns):
    import ctypes as C

    import torch
    ptrs = (C.c_void_p * 2)(own.data_ptr(), other.data_ptr())
    abi.check(abi.lib().uk_cuda_peer_barrier(ptrs, 2, 0, epoch, timeout_ns, None))
    torch.cuda.synchronize()


def test_peer_barrier_wait_expires_and_reports():
    import torch
    own = torch.zeros(8, dtype=torch.int32, device="cuda")
    other = torch.zeros(8, dtype=torch.int32, device="cuda")
    assert abi.lib().uk_cuda_pipeline_fault() == 0
    t0 = time.perf_counter()
    _peer_barrier(own, other, 1, 2_000_000)  # 2 ms; nothing posts rank 1's slot of `own`
    assert time.perf_counter() - t0 < 5.0
    assert abi.lib().uk_cuda_pipeline_fault() == 0x20
    assert abi.lib().uk_cuda_pipeline_fault() == 0
    # this rank's post landed in both arrays at its slot
    assert own[0].item() == 1 and other[0].item() == 1


def test_peer_barrier_completes_once_every_rank_posted():
    import torch
    own = torch.zeros(8, dtype=torch.int32, device="cuda")
    other = torch.zeros(8, dtype=torch.int32, device="cuda")
    own[1] = 7  # rank 1's post of epoch 7 (and of every earlier one)
    for epoch in (3, 7):
        _peer_barrier(own, other, epoch, 2_000_000_000)
        assert abi.lib().uk_cuda_pipeline_fault() == 0
    assert own[0].item() == 7 and other[0].item() == 7


def test_peer_barrier_arguments_are_checked():
    import ctypes as C

    import torch
    f = torch.zeros(8, dtype=torch.int32, device="cuda")
    ptrs = (C.c_void_p * 2)(f.data_ptr(), f.data_ptr())
    L = abi.lib()
    assert L.uk_cuda_peer_barrier(ptrs, 9, 0, 1, 10_000_000, None) == 2      # more than 8 ranks
    assert L.uk_cuda_peer_barrier(ptrs, 2, 2, 1, 10_000_000, None) == 2      # rank outside 0..n-1
    assert L.uk_cuda_peer_barrier(ptrs, 2, 0, 1, 100, None) == 2             # limit below 1 us
