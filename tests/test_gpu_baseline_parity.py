"""Parity at the BASELINE sizes themselves, with the BASELINE input
distributions, against the fp64 oracle.

* f16 GEMM 8192^3, A and B ~ N(0, 0.02) in fp16: 64 full rows
  of C plus 4096 random (i, j) elements, each against the fp64 dot product of
  the half inputs (src/codegen_hip.cpp:1851-1862 quantises to half first).
* conv N=32, 256->256, 56x56, 3x3, pad 1, channel scale, on
  both kernels (split-tf32 tensor cores and FFMA): 8 randomly chosen images
  checked in full and 4096 sampled output points of the other 24.

Two gates per case:
1. the north star's: rel_err <= 2e-2 (f16) or 1e-4 (f32) with the
   output-scale floor tau = RMS(ref) (tests/uk_testutil.py);
2. a tighter one against the reference's own algorithm on the same inputs
   (its sequential fp32 loop: src/codegen_hip.cpp:1124-1132 rounded to f16
   for the GEMM, src/reference.cpp:6-22 for the conv), so that a regression
   well inside gate 1 is still caught:
   - f16 GEMM: at most 2x the reference's error (its error is the final f16
     rounding, half an ulp; 2x allows a neighbouring f16 where the two f32
     sums straddle a rounding boundary);
   - FFMA conv: at most 4x the reference's error;
   - split-tf32 conv: at most 8x (the tensor cores' fp32 accumulator
     truncates instead of rounding, ~2e-5 of the output scale against the
     reference's ~6e-6 at this K).
"""
import numpy as np
import pytest

import unikern_b200.abi as abi
from oracle import oracle as O
from uk_testutil import F16_TOL, F32_TOL, SUM_TAU, dev, empty, host

pytestmark = pytest.mark.gpu


def _gemm_inputs(M, N, K, seed):
    rng = np.random.default_rng(seed)
    Ah = O.f32_to_f16(rng.normal(0, 0.02, (M, K)).astype(np.float32))
    Bh = O.f32_to_f16(rng.normal(0, 0.02, (K, N)).astype(np.float32))
    return Ah, Bh


def test_gemm_f16_8192_baseline_inputs_vs_f64():
    M = N = K = 8192
    Ah, Bh = _gemm_inputs(M, N, K, 8192)
    Cm = empty((M, N), "f16")
    abi.gemm_f16(dev(Ah), dev(Bh), Cm)
    got = O.f16_to_f32(host(Cm))
    assert abi.lib().uk_cuda_pipeline_fault() == 0
    assert np.isfinite(got).all()

    rng = np.random.default_rng(1)
    rows = np.unique(np.concatenate([[0, M - 1], rng.choice(M, 62, replace=False)]))
    ref_rows = O.gemm_f16_f64(Ah[rows], Bh, threads=O.nthreads())
    tau = SUM_TAU * O.rms(ref_rows)
    err_rows = O.rel_err(got[rows], ref_rows, tau)

    ij = np.stack([rng.integers(0, M, 4096), rng.integers(0, N, 4096)], axis=1)
    ref_pts = O.gemm_f16_dots_f64(Ah, Bh, ij)
    err_pts = O.rel_err(got[ij[:, 0], ij[:, 1]], ref_pts, tau)

    # the reference's own algorithm (fp32 sequential sum, one f16 rounding)
    # on the same rows: the yardstick for the tighter gate
    ref_algo = O.f16_to_f32(O.f32_to_f16(O.gemm_f16(Ah[rows], Bh, threads=O.nthreads())))
    err_algo = O.rel_err(ref_algo, ref_rows, tau)
    same = float(np.mean(got[rows] == ref_algo))
    print("8192^3 f16: rows err %.3e, points err %.3e, reference algorithm err %.3e, identical to it %.4f"
          % (err_rows, err_pts, err_algo, same))
    assert err_rows <= F16_TOL and err_pts <= F16_TOL
    assert err_rows <= 2.0 * err_algo and err_pts <= 2.0 * err_algo


@pytest.fixture(scope="module")
def conv_case():
    N, Cc, H, W, Oc = 32, 256, 56, 56, 256
    rng = np.random.default_rng(2024)
    x = rng.uniform(0, 1, (N, Cc, H, W)).astype(np.float32)
    w = rng.normal(0, np.sqrt(2.0 / (9 * Cc)), (Oc, Cc, 3, 3)).astype(np.float32)
    s = rng.uniform(0.5, 1.5, Oc).astype(np.float32)
    pick = np.random.default_rng(5)
    images = np.sort(pick.choice(N, 8, replace=False))
    ref_img = {int(n): O.conv_nchw(x[n:n + 1], w, s, 1) for n in images}
    rest = np.setdiff1d(np.arange(N), images)
    pts = np.stack([pick.choice(rest, 4096), pick.integers(0, Oc, 4096), pick.integers(0, H, 4096),
                    pick.integers(0, W, 4096)], axis=1).astype(np.int32)
    ref_pts = O.conv_nchw_points_f64(x, w, s, 1, pts)
    n0 = int(images[0])
    algo_err = O.rel_err(O.conv_nchw(x[n0:n0 + 1], w, s, 1, f32=True), ref_img[n0], SUM_TAU * O.rms(ref_img[n0]))
    return dict(x=x, w=w, s=s, images=images, ref_img=ref_img, pts=pts, ref_pts=ref_pts, algo_err=algo_err,
                shape=(N, Cc, H, W, Oc))


@pytest.mark.parametrize("path,factor", [("tensor_cores", 8.0), ("ffma", 4.0)])
def test_conv_baseline_8_images_and_sampled_points(conv_case, path, factor):
    c = conv_case
    N, Cc, H, W, Oc = c["shape"]
    y = empty((N, Oc, H, W))
    fn = abi.conv2d_tc if path == "tensor_cores" else abi.conv2d
    fn(dev(c["x"]), dev(c["w"]), y, N, H, W, Cc, 3, 3, Oc, 1, dev(c["s"]), abi.UK_CONV_NCHW)
    got = host(y)
    assert abi.lib().uk_cuda_pipeline_fault() == 0
    worst = 0.0
    for n, ref in c["ref_img"].items():
        worst = max(worst, O.rel_err(got[n:n + 1], ref, SUM_TAU * O.rms(ref)))
    tau = SUM_TAU * O.rms(next(iter(c["ref_img"].values())))
    p = c["pts"]
    err_pts = O.rel_err(got[p[:, 0], p[:, 1], p[:, 2], p[:, 3]], c["ref_pts"], tau)
    print("conv %s: 8 images err %.3e, sampled points err %.3e, reference algorithm err %.3e"
          % (path, worst, err_pts, c["algo_err"]))
    assert worst <= F32_TOL and err_pts <= F32_TOL
    assert worst <= factor * c["algo_err"] and err_pts <= factor * c["algo_err"]
