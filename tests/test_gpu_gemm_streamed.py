"""The GEMM larger than the device (scenario B, src/codegen_hip.cpp:1485-1500
of UNIKERN): B resident, A and C streamed from and to page-locked host memory
through a two-slot device ring (uk_cuda_gemm_streamed).  Every block runs the
same kernel as a device-resident GEMM of its rows, so the f16 result is
bit-identical to the resident GEMM; fp32 is held to the f64 oracle."""
import numpy as np
import pytest

import unikern_b200.abi as abi
from oracle import oracle as O
from uk_testutil import F32_TOL, SUM_TAU

pytestmark = pytest.mark.gpu


def ring_for(M, N, K, kind, rows):
    return abi.gemm_streamed_ring(M, N, K, kind, rows)


@pytest.mark.parametrize("M,N,K,rows", [(4096, 1024, 1024, 1280), (1000, 520, 264, 96), (256, 256, 64, 256),
                                        (300, 136, 72, 32)])
def test_streamed_f16_matches_resident_gemm(M, N, K, rows):
    import torch
    g = torch.Generator(device="cuda")
    g.manual_seed(M * 3 + N + K)
    A = (torch.randn((M, K), generator=g, device="cuda") * 0.5).half()
    B = (torch.randn((K, N), generator=g, device="cuda") * 0.5).half()
    ref = torch.empty((M, N), dtype=torch.float16, device="cuda")
    abi.gemm_f16(A, B, ref)
    Ah, Bh = A.cpu().pin_memory(), B.cpu().pin_memory()
    Ch = torch.full((M, N), float("nan"), dtype=torch.float16).pin_memory()
    Bd = torch.empty_like(B)
    ring = ring_for(M, N, K, 1, rows)
    for _ in range(2):  # the second call reuses the ring and the per-slot events
        abi.gemm_streamed(Ah, Bh, Ch, Bd, ring, rows)
        torch.cuda.synchronize()
        assert torch.equal(Ch, ref.cpu())
    assert abi.lib().uk_cuda_pipeline_fault() == 0


@pytest.mark.parametrize("M,N,K,rows", [(1024, 768, 512, 256), (333, 130, 257, 64)])
def test_streamed_f32_vs_f64(M, N, K, rows):
    import torch
    rng = np.random.default_rng(M + N + K)
    A = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    B = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    Ah, Bh = torch.from_numpy(A).pin_memory(), torch.from_numpy(B).pin_memory()
    Ch = torch.full((M, N), float("nan"), dtype=torch.float32).pin_memory()
    Bd = torch.empty((K, N), dtype=torch.float32, device="cuda")
    abi.gemm_streamed(Ah, Bh, Ch, Bd, ring_for(M, N, K, 0, rows), rows)
    torch.cuda.synchronize()
    ref = O.gemm_f64(A, B, threads=8)
    assert O.rel_err(Ch.numpy(), ref, SUM_TAU * O.rms(ref)) <= F32_TOL


@pytest.mark.parametrize("M,N,K,rows", [(4096, 1024, 1024, 1024), (3000, 2048, 1024, 768)])
def test_streamed_f32_tensor_cores_vs_f64_and_ffma(M, N, K, rows):
    # blocks of >= 2^30 multiply-adds take the split-tf32 tensor cores (the
    # ring then holds B^T's tf32 pairs); kind 2 forces the FFMA kernel
    import torch
    rng = np.random.default_rng(M * N + K)
    A = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    B = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    Ah, Bh = torch.from_numpy(A).pin_memory(), torch.from_numpy(B).pin_memory()
    Bd = torch.empty((K, N), dtype=torch.float32, device="cuda")
    assert abi.lib().uk_cuda_gemm_f32_prefers_tc(rows, N, K) == 1
    assert (abi.lib().uk_cuda_gemm_streamed_ring_size(M, N, K, 0, rows)
            > abi.lib().uk_cuda_gemm_streamed_ring_size(M, N, K, 2, rows) + 2 * K * N * 4)
    out = {}
    for kind, ffma in ((0, False), (2, True)):
        Ch = torch.full((M, N), float("nan"), dtype=torch.float32).pin_memory()
        abi.gemm_streamed(Ah, Bh, Ch, Bd, ring_for(M, N, K, kind, rows), rows, ffma=ffma)
        torch.cuda.synchronize()
        out[kind] = Ch.numpy().copy()
    assert abi.lib().uk_cuda_pipeline_fault() == 0
    sel = np.r_[0:64, M - 64:M]  # whole rows of the first and the last block
    ref = O.gemm_f64(A[sel], B, threads=8)
    tau = SUM_TAU * O.rms(ref)
    for kind in (0, 2):
        assert O.rel_err(out[kind][sel], ref, tau) <= F32_TOL, kind
    # both kernels agree everywhere to fp32 accuracy
    assert O.rel_err(out[0], out[2].astype(np.float64), tau) <= F32_TOL


def test_streamed_refuses_small_ring_and_pageable_memory():
    import torch
    M, N, K, rows = 512, 256, 128, 128
    Ah = torch.zeros((M, K), dtype=torch.float16).pin_memory()
    Bh = torch.zeros((K, N), dtype=torch.float16).pin_memory()
    Ch = torch.zeros((M, N), dtype=torch.float16).pin_memory()
    Bd = torch.empty((K, N), dtype=torch.float16, device="cuda")
    small = torch.empty(abi.lib().uk_cuda_gemm_streamed_ring_size(M, N, K, 1, rows) - 256, dtype=torch.uint8,
                        device="cuda")
    with pytest.raises(abi.UkError) as e:
        abi.gemm_streamed(Ah, Bh, Ch, Bd, small, rows)
    assert e.value.code == 2 and "ring" in str(e.value)
    pageable = torch.zeros((M, K), dtype=torch.float16)
    with pytest.raises(abi.UkError) as e:
        abi.gemm_streamed(pageable, Bh, Ch, Bd, ring_for(M, N, K, 1, rows), rows)
    assert e.value.code == 2 and "page-locked" in str(e.value)
