"""fp16 softmax / RMSNorm / channelscale / reduce (f16 rows, fp32 arithmetic) against
the fp64 oracle on the same half inputs (oracle/uk_oracle.c restates the
reference's cpu_softmax / cpu_rmsnorm / cpu_channelscale,
src/codegen_hip.cpp:1999-2009, :2168-2178, :2339-2344).

Gate: one f16 rounding of the fp32 result, rel_err <= 1e-3 with the floor
tau = 2^-14 (the smallest normal f16: below it f16 keeps an absolute step of
2^-24).  channelscale rounds one fp32 product, so it must equal the oracle's
fp32 product rounded to f16 bit for bit.
"""
import numpy as np
import pytest

import unikern_b200.abi as abi
from oracle import oracle as O
from uk_testutil import dev, empty, host

pytestmark = pytest.mark.gpu
F16_OUT_TOL = 1e-3
TAU = 2.0 ** -14

SHAPES = [(64, 256), (7, 33), (1, 1), (3, 4104), (8192, 4096), (2, 40000), (5, 65536), (33, 1000)]


def half(a):
    return O.f32_to_f16(np.asarray(a, np.float32))


@pytest.mark.parametrize("L,C", SHAPES)
def test_softmax_f16(L, C):
    rng = np.random.default_rng(L + C)
    Xh = half(rng.normal(0, 2, (L, C)))
    Y = empty((L, C), "f16")
    abi.softmax_f16(dev(Xh), Y)
    ref = O.softmax_f64(O.f16_to_f32(Xh))
    assert O.rel_err(O.f16_to_f32(host(Y)), ref, TAU) <= F16_OUT_TOL


@pytest.mark.parametrize("L,C", SHAPES)
def test_rmsnorm_f16(L, C):
    rng = np.random.default_rng(L * 3 + C)
    Xh = half(rng.normal(0, 1, (L, C)))
    Wh = half(rng.normal(1, 0.1, C))
    Y = empty((L, C), "f16")
    abi.rmsnorm_f16(dev(Xh), dev(Wh), Y, 1e-5)
    ref = O.rmsnorm_f64(O.f16_to_f32(Xh), O.f16_to_f32(Wh), 1e-5)
    assert O.rel_err(O.f16_to_f32(host(Y)), ref, TAU) <= F16_OUT_TOL


@pytest.mark.parametrize("L,C", SHAPES)
def test_channelscale_f16_bit_exact(L, C):
    rng = np.random.default_rng(L * 5 + C)
    Xh = half(rng.normal(0, 1, (L, C)))
    Sh = half(rng.uniform(0.5, 1.5, C))
    Y = empty((L, C), "f16")
    abi.channelscale_f16(dev(Xh), dev(Sh), Y)
    want = half(O.channelscale_f32(O.f16_to_f32(Xh), O.f16_to_f32(Sh)))
    assert np.array_equal(host(Y), want)


def test_f16_row_ops_deterministic():
    rng = np.random.default_rng(9)
    Xh = dev(half(rng.normal(0, 2, (512, 16384))))
    Y1, Y2 = empty((512, 16384), "f16"), empty((512, 16384), "f16")
    abi.softmax_f16(Xh, Y1)
    abi.softmax_f16(Xh, Y2)
    assert np.array_equal(host(Y1), host(Y2))


@pytest.mark.parametrize("rows,cols,width", [(8192, 16384, 0), (1, 1 << 24, 0), (3, 1000003, 0), (17, 7, 0),
                                             (4096, 300, 0), (2, 1 << 20, 4096), (1, 999999, 1000)])
def test_reduce_f16(rows, cols, width):
    # the widening of reduce: fp32 sums of the half inputs, one rounding
    rng = np.random.default_rng(rows + cols + width)
    Xh = half(rng.normal(0, 1, (rows, cols)))
    Y = empty((rows,), "f16")
    abi.reduce_f16(dev(Xh), Y, width)
    ref = O.f16_to_f32(Xh).astype(np.float64).sum(axis=1)
    got = O.f16_to_f32(host(Y)).astype(np.float64)
    # one binary16 rounding of a sum accurate to fp32 (floor: the sum's scale)
    tau = max(np.sqrt(cols), 1.0)
    assert np.max(np.abs(got - ref) / np.maximum(np.abs(ref), tau)) <= F16_OUT_TOL


def test_reduce_f16_exact_instance():
    # the KML verify instance: 2^20 x 2^-6 = 16384, exact in binary16
    Xh = half(np.full((1, 1 << 20), 0.015625))
    Y = empty((1,), "f16")
    abi.reduce_f16(dev(Xh), Y)
    assert O.f16_to_f32(host(Y))[0] == 16384.0
