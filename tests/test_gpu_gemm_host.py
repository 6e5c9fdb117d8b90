"""The f16 GEMM from and to host memory with the copies pipelined against the
GEMM (uk_cuda_gemm_f16_host): every row block runs the same tensor-core
kernel as a device-resident GEMM, so C must come back bit-identical to it;
pageable host memory is refused."""
import numpy as np
import pytest

import unikern_b200.abi as abi
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K,chunks", [(2048, 1024, 512, 0), (1000, 520, 264, 3), (256, 256, 64, 1),
                                          (8192, 8192, 8192, 8)])
def test_host_pipeline_matches_device_gemm(M, N, K, chunks):
    import torch
    g = torch.Generator(device="cuda")
    g.manual_seed(M + N + K)
    A = (torch.randn((M, K), generator=g, device="cuda") * 0.5).half()
    B = (torch.randn((K, N), generator=g, device="cuda") * 0.5).half()
    ref = torch.empty((M, N), dtype=torch.float16, device="cuda")
    abi.gemm_f16(A, B, ref)
    Ah, Bh = A.cpu().pin_memory(), B.cpu().pin_memory()
    Ch = torch.full((M, N), float("nan"), dtype=torch.float16).pin_memory()
    Ad, Bd, Cd = torch.empty_like(A), torch.empty_like(B), torch.empty_like(ref)
    for _ in range(2):  # the second call reuses the per-device streams and events
        abi.gemm_f16_host(Ah, Bh, Ch, Ad, Bd, Cd, chunks)
        torch.cuda.synchronize()
        assert torch.equal(Ch, ref.cpu())
    assert abi.lib().uk_cuda_pipeline_fault() == 0
    if M <= 2048:  # and against the f64 oracle of the half inputs
        a16, b16 = Ah.view(torch.int16).numpy().view(np.uint16), Bh.view(torch.int16).numpy().view(np.uint16)
        want = O.gemm_f16_f64(a16, b16)
        got = O.f16_to_f32(Ch.view(torch.int16).numpy().view(np.uint16))
        assert O.rel_err(got, want, O.rms(want)) <= 2e-2


def test_host_pipeline_refuses_pageable_memory():
    import torch
    A = torch.zeros((256, 64), dtype=torch.float16)
    B = torch.zeros((64, 256), dtype=torch.float16)
    C = torch.zeros((256, 256), dtype=torch.float16)
    Ad, Bd, Cd = A.cuda(), B.cuda(), C.cuda()
    with pytest.raises(abi.UkError) as e:
        abi.gemm_f16_host(A, B, C, Ad, Bd, Cd)
    assert e.value.code == 2 and "page-locked" in str(e.value)
