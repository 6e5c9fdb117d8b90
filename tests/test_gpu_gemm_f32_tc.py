"""The fp32 GEMM on the tcgen05 tensor cores (uk_cuda_gemm_f32_ws): split-tf32
operands, three MMAs per product, run as a 1 x 1 convolution on the
convolution's kernels.  Held to the fp32 gate against the f64 oracle, exact on
the reference's sawtooth instance (src/codegen_hip.cpp:604-605, :1030), and
checked against the FFMA kernel."""
import numpy as np
import pytest

import unikern_b200.abi as abi
from oracle import oracle as O
from uk_testutil import F32_TOL, SUM_TAU, dev, empty, host

pytestmark = pytest.mark.gpu


def tc(A, B):
    Cm = empty((A.shape[0], B.shape[1]))
    abi.gemm_f32_tc(dev(A), dev(B), Cm)
    return host(Cm)


def test_sawtooth_verify_instance_exact():
    A = O.sawtooth("A", 256 * 256).reshape(256, 256)
    B = O.sawtooth("B", 256 * 256).reshape(256, 256)
    assert np.array_equal(tc(A, B), O.gemm_f32(A, B, threads=8))


@pytest.mark.parametrize("M,N,K", [(2048, 2048, 2048), (1000, 1088, 800), (130, 64, 32), (4096, 4096, 4096),
                                   (333, 640, 2048)])
def test_tc_vs_f64(M, N, K):
    rng = np.random.default_rng(M * 5 + N * 3 + K)
    A = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    B = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    got = tc(A, B)
    rows = np.r_[0:min(M, 96), max(0, M - 32):M]
    ref = O.gemm_f64(A[rows], B, threads=8)
    tau = SUM_TAU * O.rms(ref)
    assert O.rel_err(got[rows], ref, tau) <= F32_TOL
    # and the FFMA kernel's result everywhere
    Cm = empty((M, N))
    abi.gemm_f32(dev(A), dev(B), Cm)
    assert O.rel_err(got, host(Cm).astype(np.float64), tau) <= F32_TOL
    assert abi.lib().uk_cuda_pipeline_fault() == 0


def test_workspace_and_preference_queries():
    lib = abi.lib()
    # the tf32 pairs of B^T and A, plus room for the split partial tiles
    assert lib.uk_cuda_gemm_f32_workspace_size(256, 256, 256) >= 2 * 256 * 256 * 4 * 2
    assert lib.uk_cuda_gemm_f32_workspace_size(256, 100, 256) == 0   # N % 64
    assert lib.uk_cuda_gemm_f32_workspace_size(256, 256, 100) == 0   # K % 32
    assert lib.uk_cuda_gemm_f32_prefers_tc(1024, 1024, 1024) == 1
    assert lib.uk_cuda_gemm_f32_prefers_tc(512, 512, 512) == 0


def test_shape_without_tc_is_refused_with_a_workspace():
    import torch
    A, B, Cm = empty((64, 64)), empty((64, 100)), empty((64, 100))
    ws = torch.empty(1 << 20, dtype=torch.uint8, device="cuda")
    with pytest.raises(abi.UkError) as e:
        abi.gemm_f32_tc(A, B, Cm, workspace=ws)
    assert e.value.code == 2 and "N % 64" in str(e.value)
    # without a workspace it is the FFMA GEMM
    A = np.ones((64, 64), np.float32)
    B = np.ones((64, 100), np.float32)
    Cm = empty((64, 100))
    abi.lib().uk_cuda_gemm_f32_ws(abi._p(dev(A)), abi._p(dev(B)), abi._p(Cm), 64, 100, 64, None, 0, None)
    assert np.all(host(Cm) == 64.0)
