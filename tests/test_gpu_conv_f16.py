"""fp16 convolution on the tensor cores (uk_cuda_conv2d_f16) against the fp64
oracle of the reference's cpu_conv (src/reference.cpp:6-22, restated in
oracle/uk_oracle.c) on the same half inputs.  Gate: the f16 GEMM/conv gate,
rel_err <= 2e-2 with the output-scale floor RMS(ref).  Both layouts; the
KML form reads its HWC input in place."""
import numpy as np
import pytest

import unikern_b200.abi as abi
from oracle import oracle as O
from uk_testutil import F16_TOL, dev, empty, host

pytestmark = pytest.mark.gpu


def half(a):
    return O.f32_to_f16(np.asarray(a, np.float32))


@pytest.mark.parametrize("N,Cc,H,W,Oc,K,pad,scaled", [
    (2, 64, 9, 9, 16, 3, 1, True),
    (3, 128, 13, 70, 300, 3, 1, True),
    (1, 256, 14, 14, 256, 3, 1, False),
    (2, 64, 7, 5, 40, 1, 0, True),
    (2, 192, 12, 12, 72, 3, 1, True),      # tiled pre-pass, three channel tiles, a partial hw tile
    (1, 1024, 8, 64, 64, 1, 0, False),     # a C x W plane beyond the row-staged pre-pass (tiled path only)
    (32, 256, 56, 56, 256, 3, 1, True),   # the BASELINE conv shape in fp16 (two images checked)
])
def test_conv_f16_nchw_vs_f64(N, Cc, H, W, Oc, K, pad, scaled):
    rng = np.random.default_rng(N * 100 + Cc + H)
    xh = half(rng.uniform(0, 1, (N, Cc, H, W)))
    wh = half(rng.normal(0, np.sqrt(2.0 / (K * K * Cc)), (Oc, Cc, K, K)))
    sh = half(rng.uniform(0.5, 1.5, Oc)) if scaled else None
    Ho, Wo = H + 2 * pad - K + 1, W + 2 * pad - K + 1
    y = empty((N, Oc, Ho, Wo), "f16")
    abi.conv2d_f16(dev(xh), dev(wh), y, N, H, W, Cc, K, K, Oc, pad, dev(sh) if scaled else None, abi.UK_CONV_NCHW)
    got = O.f16_to_f32(host(y))
    x32, w32 = O.f16_to_f32(xh), O.f16_to_f32(wh)
    s32 = O.f16_to_f32(sh) if scaled else None
    for n in ((0, N - 1) if N > 4 else range(N)):
        ref = O.conv_nchw(x32[n:n + 1], w32, s32, pad)
        assert O.rel_err(got[n:n + 1], ref, O.rms(ref)) <= F16_TOL
    assert abi.lib().uk_cuda_pipeline_fault() == 0


def test_conv_f16_kml_layout_in_place():
    # the KML form reads its input in place; a workspace only adds room for
    # the split partial tiles of the last round (here 14 tiles, all in it)
    H, W, Cc, Kh, Kw, Oc = 58, 58, 256, 3, 3, 256
    assert abi.lib().uk_cuda_conv2d_f16_workspace_size(1, H, W, Cc, Kh, Kw, Oc, 0, abi.UK_CONV_KML) > 0
    rng = np.random.default_rng(5)
    xh = half(rng.uniform(0, 1, H * W * Cc))
    wh = half(rng.normal(0, np.sqrt(2.0 / (9 * Cc)), Oc * Kh * Kw * Cc))
    ref = O.conv_f64(O.f16_to_f32(xh), O.f16_to_f32(wh), H, W, Cc, Kh, Kw, Oc, threads=8)
    x_d, w_d = dev(xh), dev(wh)
    y = empty((Oc * (H - 2) * (W - 2),), "f16")
    abi.conv2d_f16(x_d, w_d, y, 1, H, W, Cc, Kh, Kw, Oc, 0, None, abi.UK_CONV_KML)   # with the workspace
    assert O.rel_err(O.f16_to_f32(host(y)), ref, O.rms(ref)) <= F16_TOL
    y2 = empty((Oc * (H - 2) * (W - 2),), "f16")
    assert abi.lib().uk_cuda_conv2d_f16(x_d.data_ptr(), w_d.data_ptr(), y2.data_ptr(), 1, H, W, Cc, Kh, Kw, Oc, 0,
                                        None, abi.UK_CONV_KML, None, 0, None) == 0      # without
    assert O.rel_err(O.f16_to_f32(host(y2)), ref, O.rms(ref)) <= F16_TOL
    assert abi.lib().uk_cuda_pipeline_fault() == 0


def test_conv_f16_refuses_channel_counts_off_the_row():
    x, w, y = empty((1, 32, 8, 8), "f16"), empty((8, 32, 3, 3), "f16"), empty((1, 8, 8, 8), "f16")
    rc = abi.lib().uk_cuda_conv2d_f16(x.data_ptr(), w.data_ptr(), y.data_ptr(), 1, 8, 8, 32, 3, 3, 8, 1, None,
                                      abi.UK_CONV_NCHW, None, 0, None)
    assert rc == 2 and "multiple of 64" in abi.lib().uk_cuda_last_error().decode()
