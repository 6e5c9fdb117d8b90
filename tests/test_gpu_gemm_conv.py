"""GPU parity of the GEMMs (f32 FFMA, f16 tensor-core) and the conv through
the C ABI, against the CPU oracle (oracle/, pinned to the reference)."""
import numpy as np
import pytest

import unikern_b200.abi as abi
from oracle import oracle as O
from uk_testutil import F16_TOL, F32_TOL, SUM_TAU, dev, empty, host

pytestmark = pytest.mark.gpu


def gemm32(A, B):
    Cm = empty((A.shape[0], B.shape[1]))
    abi.gemm_f32(dev(A), dev(B), Cm)
    return host(Cm)


def gemm16(Ah, Bh):
    Cm = empty((Ah.shape[0], Bh.shape[1]), "f16")
    abi.gemm_f16(dev(Ah), dev(Bh), Cm)
    return O.f16_to_f32(host(Cm))


# ---- f32 ---------------------------------------------------------------------

def test_gemm_f32_reference_verify_instance_exact():
    # src/codegen_hip.cpp:1030 + :604-605: 256^3 sawtooth, every partial sum exact
    A = O.sawtooth("A", 256 * 256).reshape(256, 256)
    B = O.sawtooth("B", 256 * 256).reshape(256, 256)
    assert np.array_equal(gemm32(A, B), O.gemm_f32(A, B, threads=8))


@pytest.mark.parametrize("M,N,K", [(512, 512, 512), (1024, 768, 1000), (33, 47, 29), (1, 1, 1), (130, 1, 257),
                                   (3, 515, 64), (2048, 2048, 256)])
def test_gemm_f32_vs_f64(M, N, K):
    rng = np.random.default_rng(M * 7 + N * 3 + K)
    A = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    B = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    ref = O.gemm_f64(A, B, threads=8)
    tau = SUM_TAU * O.rms(ref)
    err = O.rel_err(gemm32(A, B), ref, tau)
    assert err <= F32_TOL
    # the gate is one the reference's own fp32 loop passes
    err_ref = O.rel_err(O.gemm_f32(A, B, threads=8), ref, tau)
    assert err_ref <= F32_TOL
    # and, tighter, within 4x of that loop's own error (floor 1e-6 of the
    # output scale for the shapes where the reference's sums are near exact)
    assert err <= max(4.0 * err_ref, 1e-6), (err, err_ref)


PLANS = ["128,128,1", "64,64,1", "64,64,4", "64,64,8", "32,64,1", "32,64,2", "32,64,4", "32,64,8", "32,64,1,2",
         "32,64,1,4", "32,64,1,8"]


@pytest.mark.parametrize("M,N,K", [(512, 512, 512), (300, 200, 264), (33, 47, 130)])
def test_gemm_f32_every_compiled_plan(M, N, K, monkeypatch):
    """Every compiled FFMA plan pinned through UK_SGEMM_PLAN (the vectorised
    path, and the scalar one when K is not a multiple of 4) against f64; the
    K split over warp groups of one CTA gives the same bits as the same split
    over a cluster (same K ranges, same fold order)."""
    rng = np.random.default_rng(M + N + K)
    A = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    B = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    ref = O.gemm_f64(A, B, threads=8)
    tau = SUM_TAU * O.rms(ref)
    got = {}
    for plan in PLANS:
        monkeypatch.setenv("UK_SGEMM_PLAN", plan)
        got[plan] = gemm32(A, B)
        launched = abi.last_launch()
        parts = [int(x) for x in plan.split(",")]
        if len(parts) == 4:
            assert launched["family"] == "ffma-kgroups" and launched["k_split"] == parts[3], launched
        else:
            assert launched["family"] == "ffma" and launched["tile"] == (parts[0], parts[1]), launched
            assert launched["k_split"] == parts[2], launched
        assert O.rel_err(got[plan], ref, tau) <= F32_TOL, plan
    for kg in (2, 4, 8):
        assert np.array_equal(got["32,64,1,%d" % kg], got["32,64,%d" % kg]), kg
    monkeypatch.setenv("UK_SGEMM_PLAN", "32,64,2,4")
    with pytest.raises(abi.UkError):
        gemm32(A, B)


def test_gemm_f32_k0_writes_zeros():
    Cm = empty((3, 5))
    Cm.fill_(5.0)
    abi.gemm_f32(empty((3, 0)), empty((0, 5)), Cm)
    assert np.array_equal(host(Cm), np.zeros((3, 5), np.float32))


# ---- f16 ---------------------------------------------------------------------

def test_gemm_f16_reference_verify_instance():
    # src/codegen_hip.cpp:1851-1862: sawtooth quantised to half, 256^3
    A = O.f32_to_f16(O.sawtooth("A", 256 * 256).reshape(256, 256))
    B = O.f32_to_f16(O.sawtooth("B", 256 * 256).reshape(256, 256))
    ref32 = O.gemm_f16(A, B, threads=8)
    got = gemm16(A, B)
    # the f32 sums are exact, so the only error is the final f16 rounding
    assert np.array_equal(got, O.f16_to_f32(O.f32_to_f16(ref32)))


@pytest.mark.parametrize("M,N,K", [(512, 512, 512), (256, 1024, 768), (1024, 256, 4096), (384, 640, 192),
                                   (32, 14336, 4096), (1, 4096, 4096), (33, 47, 29), (130, 72, 40)])
def test_gemm_f16_vs_f64(M, N, K):
    rng = np.random.default_rng(M + 5 * N + 11 * K)
    A = O.f32_to_f16(rng.normal(0, 0.02, (M, K)).astype(np.float32) * 25)
    B = O.f32_to_f16(rng.normal(0, 0.02, (K, N)).astype(np.float32) * 25)
    ref = O.gemm_f16_f64(A, B, threads=8)
    tau = SUM_TAU * O.rms(ref)
    err = O.rel_err(gemm16(A, B), ref, tau)
    assert err <= F16_TOL
    # tighter: within 2x of the reference algorithm's own error (fp32 sum,
    # one f16 rounding: half an f16 ulp)
    err_ref = O.rel_err(O.f16_to_f32(O.f32_to_f16(O.gemm_f16(A, B, threads=8))), ref, tau)
    assert err <= 2.0 * err_ref, (err, err_ref)


# ---- conv --------------------------------------------------------------------

def test_conv_kml_reference_verify_instance_exact():
    # src/codegen_hip.cpp:647-654: 32x32x8 input, 3x3, 16 outputs, sawtooth inits
    H, W, Cc, Kh, Kw, Oc = 32, 32, 8, 3, 3, 16
    x = O.sawtooth("A", H * W * Cc)
    w = O.sawtooth("B", Oc * Kh * Kw * Cc)
    y = empty((Oc * (H - 2) * (W - 2),))
    abi.conv2d(dev(x), dev(w), y, 1, H, W, Cc, Kh, Kw, Oc, 0, None, abi.UK_CONV_KML)
    assert np.array_equal(host(y), O.conv_f32(x, w, H, W, Cc, Kh, Kw, Oc))


@pytest.mark.parametrize("H,W,Cc,Kh,Kw,Oc", [(58, 58, 32, 3, 3, 64), (9, 7, 3, 2, 3, 5), (16, 16, 5, 1, 1, 130)])
def test_conv_kml_vs_f64(H, W, Cc, Kh, Kw, Oc):
    rng = np.random.default_rng(H * W + Cc)
    x = rng.uniform(0, 1, H * W * Cc).astype(np.float32)
    w = rng.normal(0, 0.1, Oc * Kh * Kw * Cc).astype(np.float32)
    y = empty((Oc * (H - Kh + 1) * (W - Kw + 1),))
    abi.conv2d(dev(x), dev(w), y, 1, H, W, Cc, Kh, Kw, Oc, 0, None, abi.UK_CONV_KML)
    ref = O.conv_f64(x, w, H, W, Cc, Kh, Kw, Oc, threads=8)
    assert O.rel_err(host(y), ref, SUM_TAU * O.rms(ref)) <= F32_TOL


@pytest.mark.parametrize("N,Cc,H,W,Oc,K,pad,scaled", [(2, 16, 13, 13, 24, 3, 1, True), (1, 256, 14, 14, 256, 3, 1, True),
                                                      (3, 3, 10, 11, 7, 3, 0, False), (2, 8, 9, 9, 16, 1, 0, True),
                                                      (1, 4, 6, 6, 3, 5, 2, False)])
def test_conv_nchw_vs_f64(N, Cc, H, W, Oc, K, pad, scaled):
    rng = np.random.default_rng(N * 100 + Cc + H)
    x = rng.uniform(0, 1, (N, Cc, H, W)).astype(np.float32)
    w = rng.normal(0, np.sqrt(2.0 / (K * K * Cc)), (Oc, Cc, K, K)).astype(np.float32)
    s = rng.uniform(0.5, 1.5, Oc).astype(np.float32) if scaled else None
    Ho, Wo = H + 2 * pad - K + 1, W + 2 * pad - K + 1
    y = empty((N, Oc, Ho, Wo))
    abi.conv2d(dev(x), dev(w), y, N, H, W, Cc, K, K, Oc, pad, dev(s) if scaled else None, abi.UK_CONV_NCHW)
    ref = O.conv_nchw(x, w, s, pad)
    assert O.rel_err(host(y), ref, SUM_TAU * O.rms(ref)) <= F32_TOL


@pytest.mark.parametrize("plan", ["128,128,8", "128,128,16", "64,64,8", "32,64,16"])
def test_conv_every_ffma_tile_vs_f64(plan, monkeypatch):
    """Each compiled FFMA conv tile pinned through UK_FFMA_CONV_PLAN, on a
    shape with ragged pixel and channel tiles in both layouts' NCHW form."""
    N, Cc, H, W, Oc, K, pad = 2, 24, 11, 13, 40, 3, 1
    rng = np.random.default_rng(7)
    x = rng.uniform(0, 1, (N, Cc, H, W)).astype(np.float32)
    w = rng.normal(0, np.sqrt(2.0 / (K * K * Cc)), (Oc, Cc, K, K)).astype(np.float32)
    s = rng.uniform(0.5, 1.5, Oc).astype(np.float32)
    monkeypatch.setenv("UK_FFMA_CONV_PLAN", plan)
    y = empty((N, Oc, H, W))
    abi.conv2d(dev(x), dev(w), y, N, H, W, Cc, K, K, Oc, pad, dev(s), abi.UK_CONV_NCHW)
    ref = O.conv_nchw(x, w, s, pad)
    assert O.rel_err(host(y), ref, SUM_TAU * O.rms(ref)) <= F32_TOL
    monkeypatch.setenv("UK_FFMA_CONV_PLAN", "16,16,4")
    with pytest.raises(abi.UkError):
        abi.conv2d(dev(x), dev(w), y, N, H, W, Cc, K, K, Oc, pad, dev(s), abi.UK_CONV_NCHW)


# ---- the solver's choice reaches the launcher ----------------------------------

@pytest.mark.parametrize("M,N,K,f16", [(640, 15104, 4096, True), (640, 16384, 4096, True), (512, 512, 512, False),
                                       (1024, 768, 1000, False), (4096, 4096, 4096, False)])
def test_launcher_runs_the_solver_argmin(M, N, K, f16):
    # the GEMM entry point launches the kernel family, tile and K split the
    # solver chose (uk_cuda_last_launch), and its result passes the gate
    want = abi.solve_plan(M, N, K, f16)
    rng = np.random.default_rng(M + N + K)
    rows = [0, M // 2, M - 1]
    if f16:
        A = O.f32_to_f16(rng.normal(0, 0.5, (M, K)).astype(np.float32))
        B = O.f32_to_f16(rng.normal(0, 0.5, (K, N)).astype(np.float32))
        got = gemm16(A, B)
        ref = O.gemm_f16_f64(A[rows], B, threads=8)
        tol = F16_TOL
    else:
        A = rng.uniform(-1, 1, (M, K)).astype(np.float32)
        B = rng.uniform(-1, 1, (K, N)).astype(np.float32)
        Cm = empty((M, N))
        if want["family"] == "tcgen05-2sm-3xtf32":
            abi.gemm_f32_tc(dev(A), dev(B), Cm)
        else:
            abi.gemm_f32(dev(A), dev(B), Cm)
        got = host(Cm)
        ref = O.gemm_f64(A[rows], B, threads=8)
        tol = F32_TOL
    ran = abi.last_launch()
    assert (ran["family"], ran["tile"], ran["k_split"]) == (want["family"], want["tile"], want["k_split"]), (ran, want)
    assert O.rel_err(got[rows], ref, SUM_TAU * O.rms(ref)) <= tol
