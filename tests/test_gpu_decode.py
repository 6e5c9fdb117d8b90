"""Decode-layer chain (Llama-3-8B shapes): the fused
RMSNorm -> skinny f16 GEMM kernel against the CPU oracle.

The oracle restates the chain as the reference runs it op by op: the
reference's RMSNorm in fp32 (src/codegen_hip.cpp:2168-2178, restated in
oracle/uk_oracle.c), its result rounded to f16 (the f16 GEMM's input
quantisation, :1857-1862), then the product in fp64.  Gate: the f16 GEMM's
2e-2 relative error (scale floor RMS(ref)), the tolerance every f16 GEMM test
here uses.  The fused kernel forms rms_b from split-K partial sums, so it is
not bit-identical to the op-by-op path; it must be deterministic, though.
"""
import numpy as np
import pytest

from oracle import oracle as O
from uk_testutil import F16_TOL, dev, empty, host

pytestmark = pytest.mark.gpu


def oracle_chain(X, g, Wh, eps, rows=None):
    xn = O.rmsnorm_f32(X, g, eps)
    return O.gemm_f16_f64(O.f32_to_f16(xn), Wh, rows=rows)


@pytest.mark.parametrize("B,K,N", [
    (32, 4096, 1792),    # one GPU's column block of the 8-way sharded layer
    (1, 4096, 1792),
    (7, 1024, 1000),     # ragged N, smaller cluster
    (16, 256, 136),
    (32, 64, 8),         # one k-block, one CTA per cluster
    (5, 4096, 520),      # 5 tiles: K split over a 16-CTA cluster
    (3, 200, 72),        # K not a multiple of 64: zero-filled tail
])
def test_decode_rmsnorm_gemm_matches_oracle(B, K, N):
    import torch
    rng = np.random.default_rng(B * 7 + K + N)
    X = rng.normal(0, 1, (B, K)).astype(np.float32)
    g = rng.normal(1, 0.1, K).astype(np.float32)
    Wh = O.f32_to_f16(rng.normal(0, 0.02, (K, N)).astype(np.float32))
    Y = empty((B, N), "f16")
    import unikern_b200.abi as abi
    abi.decode_rmsnorm_gemm(dev(X), dev(g), dev(Wh), Y, 1e-5)
    got = O.f16_to_f32(host(Y))
    ref = oracle_chain(X, g, Wh, 1e-5)
    err = O.rel_err(got, ref, O.rms(ref))
    assert err <= F16_TOL, err
    assert abi.lib().uk_cuda_pipeline_fault() == 0
    # deterministic: a second launch gives the same bits
    Y2 = empty((B, N), "f16")
    abi.decode_rmsnorm_gemm(dev(X), dev(g), dev(Wh), Y2, 1e-5)
    torch.cuda.synchronize()
    assert np.array_equal(host(Y2), host(Y))


def test_decode_full_layer_width_sampled():
    """B = 32 against the full 4096 x 14336 weight; 64 output columns checked."""
    import unikern_b200.abi as abi
    B, K, N = 32, 4096, 14336
    rng = np.random.default_rng(99)
    X = rng.normal(0, 1, (B, K)).astype(np.float32)
    g = rng.normal(1, 0.1, K).astype(np.float32)
    Wh = O.f32_to_f16(rng.normal(0, 0.02, (K, N)).astype(np.float32))
    Y = empty((B, N), "f16")
    abi.decode_rmsnorm_gemm(dev(X), dev(g), dev(Wh), Y, 1e-5)
    got = O.f16_to_f32(host(Y))
    cols = np.sort(rng.choice(N, 64, replace=False))
    ref = oracle_chain(X, g, np.ascontiguousarray(Wh[:, cols]), 1e-5)
    err = O.rel_err(got[:, cols], ref, O.rms(ref))
    assert err <= F16_TOL, err
    assert abi.lib().uk_cuda_pipeline_fault() == 0


@pytest.mark.parametrize("N,splits", [
    (1792, (1, 2, 3, 5, 7, 10, 16)),   # 14 tiles: one CTA per SM up to 10, two at 16
    (14336, (1, 4, 5, 6)),             # 112 tiles: four or five CTAs share an SM (shallow rings)
])
def test_decode_every_k_split_matches_oracle(N, splits, monkeypatch):
    """The K split pinned to each cluster size (UK_DECODE_KSPLIT), non-powers
    of two included: ragged k-block ranges per rank and ragged row slices in
    the distributed-shared-memory fold.  Each plan must reach the launcher
    and match the oracle on sampled columns."""
    import unikern_b200.abi as abi
    B, K = 32, 4096
    rng = np.random.default_rng(N)
    X = rng.normal(0, 1, (B, K)).astype(np.float32)
    g = rng.normal(1, 0.1, K).astype(np.float32)
    Wh = O.f32_to_f16(rng.normal(0, 0.02, (K, N)).astype(np.float32))
    cols = np.unique(np.concatenate([np.arange(0, 256), rng.choice(N, 128, replace=False), np.arange(N - 128, N)]))
    ref = oracle_chain(X, g, np.ascontiguousarray(Wh[:, cols]), 1e-5)
    Xd, gd, Wd = dev(X), dev(g), dev(Wh)
    for cs in splits:
        monkeypatch.setenv("UK_DECODE_KSPLIT", str(cs))
        Y = empty((B, N), "f16")
        abi.decode_rmsnorm_gemm(Xd, gd, Wd, Y, 1e-5)
        plan = abi.last_launch()
        assert plan["family"] == "tcgen05-skinny" and plan["k_split"] == cs, plan
        got = O.f16_to_f32(host(Y))
        err = O.rel_err(got[:, cols], ref, O.rms(ref))
        assert err <= F16_TOL, (cs, err)
        assert abi.lib().uk_cuda_pipeline_fault() == 0
    monkeypatch.delenv("UK_DECODE_KSPLIT")
    Y = empty((B, N), "f16")
    abi.decode_rmsnorm_gemm(Xd, gd, Wd, Y, 1e-5)
    assert abi.last_launch()["family"] == "tcgen05-skinny"


def test_decode_bad_shapes_are_refused():
    import unikern_b200.abi as abi
    X = empty((33, 64))
    g = empty((64,))
    W = empty((64, 64), "f16")
    Y = empty((33, 64), "f16")
    with pytest.raises(abi.UkError):
        abi.decode_rmsnorm_gemm(X, g, W, Y)          # B > 32
    with pytest.raises(abi.UkError):
        abi.decode_rmsnorm_gemm(empty((4, 100)), empty((100,)), empty((100, 64), "f16"), empty((4, 64), "f16"))  # K % 8
    ws = abi.decode_workspace(4, 64)
    with pytest.raises(abi.UkError):  # workspace too small for B=32
        abi.decode_rmsnorm_gemm(empty((32, 64)), empty((64,)), empty((64, 64), "f16"), empty((32, 64), "f16"),
                                workspace=ws)
