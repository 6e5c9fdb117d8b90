"""The tensor-core convolution (uk_cuda_conv2d_f32_ws: split-tf32 operands on
tcgen05) against the fp64 oracle of the reference's cpu_conv
(src/reference.cpp:6-22, restated in oracle/uk_oracle.c), with the same fp32
gate as the FFMA kernel: rel_err <= 1e-4 with the output-scale floor.

Shapes cover both layouts, channel counts that are multiples of 32 (the
tensor-core path), output widths above the 64-pixel tile, more than 256
output channels (two channel tiles), 1x1 and 3x3 filters, padding 0 and 1,
and the KML BASELINE declaration (the full NCHW BASELINE batch is in
tests/test_gpu_baseline_parity.py).  Shapes the tensor cores do not take
(C not a multiple of 32) must run the FFMA kernel and give its bits.
"""
import numpy as np
import pytest

import unikern_b200.abi as abi
from oracle import oracle as O
from uk_testutil import F32_TOL, SUM_TAU, dev, empty, host

pytestmark = pytest.mark.gpu


def run_nchw(x, w, s, pad, tc=True):
    N, Cc, H, W = x.shape
    Oc, _, Kh, Kw = w.shape
    y = empty((N, Oc, H + 2 * pad - Kh + 1, W + 2 * pad - Kw + 1))
    fn = abi.conv2d_tc if tc else abi.conv2d
    fn(dev(x), dev(w), y, N, H, W, Cc, Kh, Kw, Oc, pad, dev(s) if s is not None else None, abi.UK_CONV_NCHW)
    return host(y)


@pytest.mark.parametrize("N,Cc,H,W,Oc,K,pad,scaled", [
    (2, 32, 9, 9, 16, 3, 1, True),
    (3, 64, 13, 70, 300, 3, 1, True),     # two w tiles, two channel tiles
    (1, 256, 14, 14, 256, 3, 1, True),
    (2, 96, 7, 5, 40, 1, 0, False),        # 1x1
    (2, 96, 8, 10, 40, 3, 1, True),        # tiled pre-pass with a partial channel tile (H*W % 4 == 0)
    (1, 32, 6, 66, 8, 3, 0, True),         # valid padding, ragged tiles
    (1, 64, 20, 20, 64, 5, 2, False),      # 5x5, pad 2
])
def test_conv_tc_nchw_vs_f64(N, Cc, H, W, Oc, K, pad, scaled):
    rng = np.random.default_rng(N * 1000 + Cc * 10 + H)
    x = rng.uniform(0, 1, (N, Cc, H, W)).astype(np.float32)
    w = rng.normal(0, np.sqrt(2.0 / (K * K * Cc)), (Oc, Cc, K, K)).astype(np.float32)
    s = rng.uniform(0.5, 1.5, Oc).astype(np.float32) if scaled else None
    assert abi.lib().uk_cuda_conv2d_workspace_size(N, H, W, Cc, K, K, Oc, pad, abi.UK_CONV_NCHW) > 0
    got = run_nchw(x, w, s, pad)
    ref = O.conv_nchw(x, w, s, pad)
    assert O.rel_err(got, ref, SUM_TAU * O.rms(ref)) <= F32_TOL
    assert abi.lib().uk_cuda_pipeline_fault() == 0
    # and against the FFMA kernel of the same op
    ffma = run_nchw(x, w, s, pad, tc=False)
    assert O.rel_err(got, ffma.astype(np.float64), SUM_TAU * O.rms(ref)) <= F32_TOL


def test_conv_tc_last_round_split_matches_unsplit():
    # the size query's workspace lets the last round of tiles split along K;
    # a workspace holding only the operand pairs runs it unsplit
    import torch
    N, Cc, H, W, Oc, pad = 3, 128, 28, 28, 96, 1
    rng = np.random.default_rng(77)
    x = rng.uniform(0, 1, (N, Cc, H, W)).astype(np.float32)
    w = rng.normal(0, np.sqrt(2.0 / (9 * Cc)), (Oc, Cc, 3, 3)).astype(np.float32)
    full = abi.lib().uk_cuda_conv2d_workspace_size(N, H, W, Cc, 3, 3, Oc, pad, abi.UK_CONV_NCHW)
    base = 2 * (-(-N * H * W * Cc * 4 // 256) * 256) + 2 * (-(-Oc * 9 * Cc * 4 // 256) * 256)
    assert full > base
    out = []
    for nbytes in (full, base):
        ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
        y = empty((N, Oc, H, W))
        abi.check(abi.lib().uk_cuda_conv2d_f32_ws(dev(x).data_ptr(), dev(w).data_ptr(), y.data_ptr(), N, H, W, Cc, 3,
                                                  3, Oc, pad, None, abi.UK_CONV_NCHW, ws.data_ptr(), nbytes, None))
        out.append(host(y))
    ref = O.conv_nchw(x, w, None, pad)
    for got in out:
        assert O.rel_err(got, ref, SUM_TAU * O.rms(ref)) <= F32_TOL
    # the two group the k-steps differently in the tensor cores' accumulator
    # (its truncation error is ~2e-5 of the output scale): fp32-gate close
    assert O.rel_err(out[0], out[1].astype(np.float64), SUM_TAU * O.rms(ref)) <= F32_TOL
    assert abi.lib().uk_cuda_pipeline_fault() == 0


def test_conv_tc_kml_layout_vs_f64():
    # the KML conv contract at its BASELINE declaration: [58, 58, 256, 3, 3, 256]
    H, W, Cc, Kh, Kw, Oc = 58, 58, 256, 3, 3, 256
    rng = np.random.default_rng(58)
    x = rng.uniform(0, 1, H * W * Cc).astype(np.float32)
    w = rng.normal(0, np.sqrt(2.0 / (9 * Cc)), Oc * Kh * Kw * Cc).astype(np.float32)
    y = empty((Oc * (H - 2) * (W - 2),))
    abi.conv2d_tc(dev(x), dev(w), y, 1, H, W, Cc, Kh, Kw, Oc, 0, None, abi.UK_CONV_KML)
    ref = O.conv_f64(x, w, H, W, Cc, Kh, Kw, Oc, threads=8)
    assert O.rel_err(host(y), ref, SUM_TAU * O.rms(ref)) <= F32_TOL


def test_conv_tc_sawtooth_instance_exact():
    # the reference's exact operands (multiples of 2^-4): every product and
    # partial sum is exact, so the split path must reproduce fp32 bit for bit
    H, W, Cc, Kh, Kw, Oc = 34, 34, 32, 3, 3, 16
    x = O.sawtooth("A", H * W * Cc)
    w = O.sawtooth("B", Oc * Kh * Kw * Cc)
    y = empty((Oc * (H - 2) * (W - 2),))
    abi.conv2d_tc(dev(x), dev(w), y, 1, H, W, Cc, Kh, Kw, Oc, 0, None, abi.UK_CONV_KML)
    assert np.array_equal(host(y), O.conv_f32(x, w, H, W, Cc, Kh, Kw, Oc))


def test_conv_tc_other_shapes_take_the_ffma_kernel():
    N, Cc, H, W, Oc = 2, 8, 9, 9, 16
    assert abi.lib().uk_cuda_conv2d_workspace_size(N, H, W, Cc, 3, 3, Oc, 1, abi.UK_CONV_NCHW) == 0
    rng = np.random.default_rng(3)
    x = rng.uniform(0, 1, (N, Cc, H, W)).astype(np.float32)
    w = rng.normal(0, 0.2, (Oc, Cc, 3, 3)).astype(np.float32)
    assert np.array_equal(run_nchw(x, w, None, 1), run_nchw(x, w, None, 1, tc=False))


def test_conv_tc_missing_workspace_is_refused():
    x, w, y = empty((1, 32, 8, 8)), empty((8, 32, 3, 3)), empty((1, 8, 8, 8))
    rc = abi.lib().uk_cuda_conv2d_f32_ws(x.data_ptr(), w.data_ptr(), y.data_ptr(), 1, 8, 8, 32, 3, 3, 8, 1, None,
                                         abi.UK_CONV_NCHW, None, 0, None)
    assert rc == 2 and "workspace" in abi.lib().uk_cuda_last_error().decode()


# ---- the conv from and to host memory (uk_cuda_conv2d_f32_host) ----------------------

@pytest.mark.parametrize("N,Cc,H,W,Oc,K,pad,chunks,scaled", [
    (7, 64, 13, 20, 48, 3, 1, 3, True),     # ragged last block (3 + 3 + 1 images)
    (4, 32, 9, 9, 16, 1, 0, 0, False),       # default 8 chunks: one image per block, no scale
    (5, 40, 8, 8, 24, 3, 1, 2, True),        # C % 32 != 0: each block runs the FFMA kernel
])
def test_conv_host_equals_the_device_op(N, Cc, H, W, Oc, K, pad, chunks, scaled):
    """Blocks of images through the host pipeline match the same convolution
    run on the whole batch on the device, and the f64 oracle."""
    import torch
    rng = np.random.default_rng(N * 31 + Cc + H)
    x = rng.uniform(0, 1, (N, Cc, H, W)).astype(np.float32)
    w = rng.normal(0, np.sqrt(2.0 / (K * K * Cc)), (Oc, Cc, K, K)).astype(np.float32)
    s = rng.uniform(0.5, 1.5, Oc).astype(np.float32) if scaled else None
    Ho, Wo = H + 2 * pad - K + 1, W + 2 * pad - K + 1
    pin = lambda a: torch.from_numpy(a).pin_memory()  # noqa: E731
    xh, wh = pin(x), pin(w)
    sh = pin(s) if scaled else None
    yh = torch.full((N, Oc, Ho, Wo), float("nan")).pin_memory()
    xd, wd = empty(x.shape), empty(w.shape)
    sd = empty((Oc,)) if scaled else None
    yd = empty((N, Oc, Ho, Wo))
    abi.conv2d_host(xh, wh, sh, yh, xd, wd, sd, yd, N, H, W, Cc, K, K, Oc, pad, chunks)
    torch.cuda.synchronize()
    got = yh.numpy()
    ref = O.conv_nchw(x, w, s, pad)
    assert O.rel_err(got, ref, SUM_TAU * O.rms(ref)) <= F32_TOL
    whole = run_nchw(x, w, s, pad)
    assert O.rel_err(got, whole.astype(np.float64), SUM_TAU * O.rms(ref)) <= F32_TOL
    assert abi.lib().uk_cuda_pipeline_fault() == 0


def test_conv_host_refuses_a_half_given_scale():
    import torch
    x, w, y = empty((1, 32, 4, 4)), empty((8, 32, 1, 1)), empty((1, 8, 4, 4))
    xh, wh = torch.zeros((1, 32, 4, 4)).pin_memory(), torch.zeros((8, 32, 1, 1)).pin_memory()
    yh = torch.zeros((1, 8, 4, 4)).pin_memory()
    sh = torch.ones(8).pin_memory()
    with pytest.raises(abi.UkError):
        abi.conv2d_host(xh, wh, sh, yh, x, w, None, y, 1, 4, 4, 32, 1, 1, 8, 0, 1)
