"""GPU parity of the HBM-bound ops (channelscale, reduce, RMSNorm, softmax)
through the C ABI, against the CPU oracle (oracle/, pinned to the reference).
"""
import numpy as np
import pytest

import unikern_b200.abi as abi
from oracle import oracle as O
from uk_testutil import F32_TOL, SUM_TAU, dev, empty, host, torch

pytestmark = pytest.mark.gpu


# ---- channelscale: bit-exact (one fp32 multiply per element) ----------------

@pytest.mark.parametrize("L,C", [(64, 256), (65536, 256), (7, 33), (1, 1), (3, 4099), (1000, 4),
                                 (8192, 16384), (5, 2048), (3, 32768), (2, 40000), (9, 6000)])
def test_channelscale_bit_exact(L, C):
    rng = np.random.default_rng(L * 7 + C)
    X = rng.normal(0, 1, (L, C)).astype(np.float32)
    S = rng.uniform(0.5, 1.5, C).astype(np.float32)
    Y = empty((L, C))
    abi.channelscale(dev(X), dev(S), Y)
    assert np.array_equal(host(Y), O.channelscale_f32(X, S))


def test_channelscale_reference_verify_instance():
    # src/codegen_hip.cpp:2378-2380: initX / initS sawtooth at the sample shape
    L, C = 65536, 256
    X = O.sawtooth("A", L * C).reshape(L, C)
    S = O.sawtooth("W", C)
    Y = empty((L, C))
    abi.channelscale(dev(X), dev(S), Y)
    assert np.array_equal(host(Y), O.channelscale_f32(X, S))


def test_channelscale_misaligned_pointer_scalar_path():
    t = torch()
    L, C = 5, 64
    X = np.random.default_rng(1).normal(0, 1, (L, C + 1)).astype(np.float32)
    S = np.linspace(0.5, 1.5, C + 1).astype(np.float32)
    dX, dS = dev(X), dev(S)
    Y = t.zeros((L, C + 1), device="cuda")
    # views that start one float in: 4-byte aligned, not 16-byte aligned
    x1 = dX.view(-1)[1:1 + L * C]
    s1 = dS[1:1 + C]
    y1 = Y.view(-1)[1:1 + L * C]
    abi.check(abi.lib().uk_cuda_channelscale_f32(x1.data_ptr(), s1.data_ptr(), y1.data_ptr(), L, C,
                                                 t.cuda.current_stream().cuda_stream))
    want = O.channelscale_f32(X.reshape(-1)[1:1 + L * C].reshape(L, C), S[1:])
    assert np.array_equal(host(y1).reshape(L, C), want)


# ---- reduce ------------------------------------------------------------------

def run_reduce(X):
    t = torch()
    rows, cols = X.shape
    Y = empty((rows,))
    ws_bytes = abi.reduce_workspace_size(rows, cols)
    ws = t.empty(max(1, ws_bytes // 4), dtype=t.float32, device="cuda") if ws_bytes else None
    abi.reduce(dev(X), Y, ws)
    return host(Y)


def test_reduce_reference_verify_instance_exact():
    # src/codegen_hip.cpp:921-924: 2^20 values of 2^-6 sum to 16384 in any order
    X = np.full((1, 1 << 20), 0.015625, np.float32)
    assert run_reduce(X)[0] == 16384.0
    X = np.full((1, 1 << 24), 0.015625, np.float32)
    assert run_reduce(X)[0] == 262144.0


@pytest.mark.parametrize("rows,cols", [(8192, 16384), (1, 134217728 // 8), (1, 1000003), (3, 5000001),
                                       (4096, 300), (17, 1), (1, 7), (100, 4096)])
def test_reduce_vs_f64(rows, cols):
    X = np.random.default_rng(rows + cols).normal(0, 1, (rows, cols)).astype(np.float32)
    got = run_reduce(X)
    ref = O.row_reduce_f64(X)
    tau = SUM_TAU * max(O.rms(ref), np.sqrt(cols))
    assert O.rel_err(got, ref, tau) <= F32_TOL


def test_reduce_deterministic_and_matches_blocked_basis():
    X = np.random.default_rng(9).normal(0, 1, (1, 1 << 22)).astype(np.float32)
    a, b = run_reduce(X), run_reduce(X)
    assert np.array_equal(a, b)
    basis = O.reduce_blocked_f32(X[0], 1024)  # the reference's differential basis
    assert abs(a[0] - basis) / max(abs(basis), 1e-6) <= 0.03125


@pytest.mark.parametrize("width", [256, 1000, 4096, 1 << 20, (1 << 20) + 7])
def test_reduce_pinned_width(width):
    # the UK_REDUCE_WIDTH knob: any pass-1 width gives the exact verify sum,
    # and the f64 gate on random rows
    X = np.full((1, 1 << 20), 0.015625, np.float32)
    Y = empty((1,))
    abi.reduce_width(dev(X), Y, width)
    assert host(Y)[0] == 16384.0
    R = np.random.default_rng(width).normal(0, 1, (3, 1000003)).astype(np.float32)
    Y = empty((3,))
    abi.reduce_width(dev(R), Y, width)
    ref = O.row_reduce_f64(R)
    assert O.rel_err(host(Y), ref, SUM_TAU * max(O.rms(ref), 1000.0)) <= F32_TOL


def test_reduce_alternating_wide_range():
    # tests/acceptance.cpp:1555-1608: the parallel sum must be at least as close
    # to the exact f64 sum as the reference's blocked basis
    n = 1 << 24
    X = np.where(np.arange(n) % 2 == 1, np.float32(1e-6), np.float32(1e6)).astype(np.float32)[None]
    exact = O.reduce_f64(X)
    got = run_reduce(X)[0]
    basis = O.reduce_blocked_f32(X[0], 1024)
    assert abs(got - exact) <= abs(basis - exact) + 1e-7 * abs(exact)


def test_reduce_zero_columns_writes_zero():
    t = torch()
    Y = t.full((5,), 7.0, device="cuda")
    abi.check(abi.lib().uk_cuda_reduce_f32(None, Y.data_ptr(), 5, 0, None, 0, t.cuda.current_stream().cuda_stream))
    assert host(Y).tolist() == [0.0] * 5


def test_reduce_missing_workspace_is_refused():
    rows, cols = 1, 1 << 22
    need = abi.reduce_workspace_size(rows, cols)
    assert need > 0
    X = empty((rows, cols))
    Y = empty((rows,))
    with pytest.raises(abi.UkError) as e:
        abi.reduce(X, Y, None)
    assert e.value.code == 2


# ---- rmsnorm -----------------------------------------------------------------

def test_rmsnorm_reference_verify_instance():
    # src/codegen_hip.cpp:2212-2214: initX / initW, eps 1e-6, shape of the sample
    L, C = 65536, 256
    X = O.sawtooth("A", L * C).reshape(L, C)
    W = O.sawtooth("W", C)
    Y = empty((L, C))
    abi.rmsnorm(dev(X), dev(W), Y, 1e-6)
    got = host(Y)
    assert O.ref_rel(got, O.rmsnorm_f32(X, W, 1e-6)) <= 1e-6  # the reference gate is 2^-5
    assert O.rel_err(got, O.rmsnorm_f64(X, W, 1e-6), 1e-30) <= F32_TOL


@pytest.mark.parametrize("L,C,eps", [(8192, 16384, 1e-5), (32, 4096, 1e-5), (1, 4096, 1e-6), (300, 1000, 1e-5),
                                     (7, 333, 1e-6), (5, 40000, 1e-5), (3, 1, 1e-6), (2, 70001, 1e-5)])
def test_rmsnorm_vs_f64(L, C, eps):
    rng = np.random.default_rng(L * 31 + C)
    X = rng.normal(0, 1, (L, C)).astype(np.float32)
    W = rng.normal(1, 0.1, C).astype(np.float32)
    Y = empty((L, C))
    abi.rmsnorm(dev(X), dev(W), Y, eps)
    assert O.rel_err(host(Y), O.rmsnorm_f64(X, W, eps), 1e-30) <= F32_TOL


# ---- softmax -----------------------------------------------------------------

def test_softmax_reference_verify_instance():
    L, C = 65536, 256
    X = O.sawtooth("A", L * C).reshape(L, C)
    Y = empty((L, C))
    abi.softmax(dev(X), Y)
    got = host(Y)
    assert O.ref_rel(got, O.softmax_f32(X)) <= 1e-5
    assert O.rel_err(got, O.softmax_f64(X), 1e-30) <= F32_TOL


@pytest.mark.parametrize("L,C", [(8192, 16384), (256, 8192), (32, 8192), (1, 256), (9, 333), (4, 40000),
                                 (2, 70001), (5, 1)])
def test_softmax_vs_f64(L, C):
    X = np.random.default_rng(L * 13 + C).normal(0, 2, (L, C)).astype(np.float32)
    Y = empty((L, C))
    abi.softmax(dev(X), Y)
    got = host(Y)
    assert O.rel_err(got, O.softmax_f64(X), 1e-30) <= F32_TOL
    assert np.allclose(got.astype(np.float64).sum(axis=1), 1.0, atol=1e-4)


# ---- residency refusal (the reference's oversubscription signal) -------------

def test_host_pointer_refused_with_code_5():
    t = torch()
    Xh = t.zeros((4, 4)).pin_memory()
    Y = empty((4, 4))
    S = empty((4,))
    rc = abi.lib().uk_cuda_channelscale_f32(Xh.data_ptr(), S.data_ptr(), Y.data_ptr(), 4, 4,
                                            t.cuda.current_stream().cuda_stream)
    assert rc == 5
    assert "device-resident" in abi.lib().uk_cuda_last_error().decode()


# ---- the row ops from and to host memory (uk_cuda_rowop_host) -------------------------

@pytest.mark.parametrize("op", ["softmax", "rmsnorm", "channelscale", "reduce"])
@pytest.mark.parametrize("L,C,chunks", [(1024, 4096, 0), (1000, 1000, 7), (5, 2048, 8), (3, 100, 1)])
def test_rowop_host_equals_the_device_op(op, L, C, chunks):
    # rows are independent and each block runs the same per-row plan, so the
    # pipelined host-to-host call gives the device op's bits
    import torch
    rng = np.random.default_rng(L + C + chunks)
    X = rng.normal(0, 2.0, (L, C)).astype(np.float32)
    W = rng.normal(1, 0.1, C).astype(np.float32)
    Xd, Wd = dev(X), dev(W)
    want = empty((L,)) if op == "reduce" else empty((L, C))
    if op == "softmax":
        abi.softmax(Xd, want)
    elif op == "rmsnorm":
        abi.rmsnorm(Xd, Wd, want, 1e-5)
    elif op == "channelscale":
        abi.channelscale(Xd, Wd, want)
    else:
        abi.reduce(Xd, want)
    Xh, Wh = torch.from_numpy(X).pin_memory(), torch.from_numpy(W).pin_memory()
    Yh = torch.empty(tuple(want.shape)).pin_memory()
    Xs, Ws, Ys = torch.empty_like(Xd), torch.empty_like(Wd), torch.empty_like(want)
    abi.rowop_host(op, Xh, Wh, Yh, Xs, Ws, Ys, 1e-5, chunks)
    torch.cuda.synchronize()
    assert np.array_equal(Yh.numpy(), host(want))
