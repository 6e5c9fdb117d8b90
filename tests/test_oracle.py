"""Pin the CPU oracle before trusting it (CPU only).

1. The reference's own known-answer tests (tests/acceptance.cpp of UNIKERN),
   restated against the oracle.
2. The golden vectors in tests/golden/reference_vectors.npz, produced by the
   reference's own code (tests/golden/make_golden.py): bit-exact.
3. Where the reference-compiled checker exists (oracle/_ref, built only in a
   container holding the reference tree), the oracle against it on fresh
   seeded inputs: bit-exact.
"""
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O

GOLD = np.load(Path(__file__).parent / "golden" / "reference_vectors.npz")


# ---- 1. known-answer tests: tests/acceptance.cpp:1322-1356 -------------------

def test_conv_kat_1x1():
    y = O.conv_f32(np.array([1, 2, 3, 4], np.float32), np.array([0.5], np.float32), 2, 2, 1, 1, 1, 1)
    assert y.tolist() == [0.5, 1.0, 1.5, 2.0]


def test_conv_kat_identity_trace():
    x = np.arange(1, 10, dtype=np.float32)
    w = np.array([1, 0, 0, 0, 1, 0, 0, 0, 1], np.float32)
    assert O.conv_f32(x, w, 3, 3, 1, 3, 3, 1).tolist() == [15.0]


def test_conv_kat_multichannel():
    y = O.conv_f32(np.array([1, 2, 3, 4], np.float32), np.array([1, 10, -1, 1], np.float32), 1, 2, 2, 1, 1, 2)
    assert y.tolist() == [21.0, 43.0, 1.0, 1.0]


def test_reduce_kat_exact_and_empty():
    v = np.full(1 << 20, 0.015625, np.float32)
    assert O.reduce_f32(v) == 16384.0
    assert O.reduce_f32(v[:0]) == 0.0
    assert O.reduce_blocked_f32(v, 1024) == 16384.0


def test_reduce_kat_basis_2p24():
    # tests/acceptance.cpp:2334-2348: blocked == sequential == 262144 at 2^24
    v = np.full(1 << 24, 0.015625, np.float32)
    assert O.reduce_f32(v) == 262144.0 and O.reduce_blocked_f32(v, 1024) == 262144.0


def test_reduce_order_arm():
    # tests/acceptance.cpp:1555-1608: two-pass is >= 10x closer to the f64 sum
    n = 1 << 20
    x = np.where(np.arange(n) % 2 == 1, np.float32(1e-6), np.float32(1e6)).astype(np.float32)
    exact = float(np.sum(x.astype(np.float64)))
    seq = O.reduce_f32(x)
    two = O.reduce_blocked_f32(x, 1024)
    seq_err = abs(seq - exact) / abs(exact)
    two_err = abs(two - exact) / abs(exact)
    assert seq_err > 1e-4 and two_err < seq_err / 10
    assert abs(two - seq) / abs(seq) <= 0.03125


def test_tolerance_table():
    import json
    d = json.loads((Path(__file__).parent / "golden" / "kml_contract.json").read_text())
    assert d["tolerance"] == {"fp32": 0.03125, "fp16": 0.0625, "int8": 0.0}


# ---- 2. golden vectors from the reference itself -----------------------------

def test_golden_initialisers():
    n = GOLD["initA"].size
    assert np.array_equal(O.sawtooth("A", n), GOLD["initA"])
    assert np.array_equal(O.sawtooth("B", n), GOLD["initB"])
    assert np.array_equal(O.sawtooth("A", n), GOLD["initX"])  # initX is the initA sawtooth
    assert np.array_equal(O.sawtooth("W", n), GOLD["initW"])
    assert np.array_equal(O.sawtooth("W", n), GOLD["initS"])


def test_golden_gemm_f32():
    assert np.array_equal(O.gemm_f32(GOLD["gemm_A"], GOLD["gemm_B"]), GOLD["gemm_C"])
    As = GOLD["initA"][:4096].reshape(64, 64)
    Bs = GOLD["initB"][:4096].reshape(64, 64)
    assert np.array_equal(O.gemm_f32(As, Bs), GOLD["gemm_saw_C"])


def test_golden_gemm_f16():
    assert np.array_equal(O.gemm_f16(GOLD["gemm_f16_A"], GOLD["gemm_f16_B"]), GOLD["gemm_f16_C"])


def test_golden_conv():
    H, W, Cc, Kh, Kw, Oc = GOLD["conv_dims"].tolist()
    y = O.conv_f32(GOLD["conv_x"], GOLD["conv_w"], H, W, Cc, Kh, Kw, Oc, threads=2)
    assert np.array_equal(y, GOLD["conv_y"])


def test_golden_conv_nchw_matches_padded_hwc():
    # the NCHW/pad form equals the reference's valid HWC conv on a host-padded input
    H, W, Cc, Kh, Kw, Oc = GOLD["conv_dims"].tolist()
    x, w = GOLD["conv_x"], GOLD["conv_w"]
    pad = 1
    xp = np.zeros((H + 2, W + 2, Cc), np.float32)
    xp[1:-1, 1:-1] = x
    ref = O.conv_f32(xp, w, H + 2, W + 2, Cc, Kh, Kw, Oc)
    x_nchw = x.transpose(2, 0, 1)[None]
    w_nchw = w.transpose(0, 3, 1, 2)
    y = O.conv_nchw(x_nchw, w_nchw, None, pad, f32=True, threads=1)
    assert np.array_equal(y.reshape(-1), ref)


def test_golden_reduce():
    seq = [O.reduce_f32(GOLD["reduce_x"]), O.reduce_f32(GOLD["reduce_alt"])]
    blk = [O.reduce_blocked_f32(GOLD["reduce_x"], 1024), O.reduce_blocked_f32(GOLD["reduce_alt"], 1024)]
    assert np.array_equal(np.array(seq, np.float32), GOLD["reduce_seq"])
    assert np.array_equal(np.array(blk, np.float32), GOLD["reduce_blk"][:2])
    assert np.float32(blk[0]) == GOLD["reduce_blk"][2]  # the emitted program's basis


def test_golden_row_reduce_rows_equal_scalar():
    x = GOLD["reduce_x"][:10000].reshape(10, 1000)
    y = O.row_reduce_f32(x, 1024, threads=3)
    assert all(np.float32(O.reduce_blocked_f32(x[i], 1024)) == y[i] for i in range(10))


def test_golden_softmax():
    assert np.array_equal(O.softmax_f32(GOLD["softmax_X"], threads=2), GOLD["softmax_Y"])


def test_golden_rmsnorm():
    assert np.array_equal(O.rmsnorm_f32(GOLD["rmsnorm_X"], GOLD["rmsnorm_W"], 1e-6), GOLD["rmsnorm_Y"])


def test_golden_channelscale():
    assert np.array_equal(O.channelscale_f32(GOLD["channelscale_X"], GOLD["channelscale_S"]),
                          GOLD["channelscale_Y"])


def test_thread_count_invariance():
    rng = np.random.default_rng(3)
    A = rng.uniform(-1, 1, (40, 33)).astype(np.float32)
    B = rng.uniform(-1, 1, (33, 21)).astype(np.float32)
    assert np.array_equal(O.gemm_f32(A, B, threads=1), O.gemm_f32(A, B, threads=4))
    X = rng.normal(0, 2, (17, 130)).astype(np.float32)
    assert np.array_equal(O.softmax_f32(X, threads=1), O.softmax_f32(X, threads=5))


def test_f64_twins_close_to_f32():
    rng = np.random.default_rng(4)
    A = rng.uniform(-1, 1, (20, 50)).astype(np.float32)
    B = rng.uniform(-1, 1, (50, 30)).astype(np.float32)
    r64 = O.gemm_f64(A, B)
    assert O.rel_err(O.gemm_f32(A, B), r64, 1e-3 * O.rms(r64)) < 1e-5
    assert np.allclose(r64, A.astype(np.float64) @ B.astype(np.float64), rtol=1e-12, atol=1e-12)


def test_half_conversion_rne():
    vals = np.array([0.1, 1 + 2 ** -11, 1 + 3 * 2 ** -11, 65504, 65520, -2 ** -24, 2 ** -25, 1e-8], np.float32)
    h = O.f32_to_f16(vals)
    with np.errstate(over="ignore"):
        want = vals.astype(np.float16)
    assert np.array_equal(h, want.view(np.uint16))
    assert np.array_equal(O.f16_to_f32(h), want.astype(np.float32))


# ---- 3. live reference, where oracle/_ref was built ---------------------------

needs_ref = pytest.mark.skipif(O.emit() is None or O.ref() is None,
                               reason="reference-compiled checker not built here")


@needs_ref
@pytest.mark.parametrize("seed", [0, 1, 2])
def test_live_reference_conv_and_reduce(seed):
    rng = np.random.default_rng(100 + seed)
    H, W, Cc, Kh, Kw, Oc = 7 + seed, 6 + 2 * seed, 1 + seed, 1 + seed, 2 + seed % 2, 3
    x = rng.normal(0, 1, H * W * Cc).astype(np.float32)
    w = rng.normal(0, 1, Oc * Kh * Kw * Cc).astype(np.float32)
    y = np.zeros(Oc * (H - Kh + 1) * (W - Kw + 1), np.float32)
    O.ref().ref_cpu_conv(x, w, y, H, W, Cc, Kh, Kw, Oc)
    assert np.array_equal(O.conv_f32(x, w, H, W, Cc, Kh, Kw, Oc), y)
    v = rng.normal(0, 1, 5000 + 777 * seed).astype(np.float32)
    assert np.float32(O.reduce_f32(v)) == O.ref().ref_cpu_reduce(v, v.size)
    for width in (0, 1, 1024, 4096):
        assert np.float32(O.reduce_blocked_f32(v, width)) == O.ref().ref_cpu_reduce_blocked(v, v.size, width)


@needs_ref
@pytest.mark.parametrize("seed", [0, 1])
def test_live_reference_emitted_cpu_refs(seed):
    e = O.emit()
    rng = np.random.default_rng(200 + seed)
    M, N, K = 19 + seed, 23, 41 + 3 * seed
    A = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    B = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    Cm = np.zeros((M, N), np.float32)
    e.emit_gemm_cpu_ref(A, B, Cm, M, N, K)
    assert np.array_equal(O.gemm_f32(A, B), Cm)
    Ah = O.f32_to_f16(A)
    Bh = O.f32_to_f16(B)
    e.emit_gemm_f16_cpu_ref(O.f16_to_f32(Ah), O.f16_to_f32(Bh), Cm, M, N, K)
    assert np.array_equal(O.gemm_f16(Ah, Bh), Cm)
    X = rng.normal(0, 2, (9, 333)).astype(np.float32)
    Y = np.zeros_like(X)
    e.emit_softmax(X, Y, 9, 333)
    assert np.array_equal(O.softmax_f32(X), Y)
    Wg = rng.normal(1, 0.1, 333).astype(np.float32)
    e.emit_rmsnorm(X, Wg, Y, 9, 333)
    assert np.array_equal(O.rmsnorm_f32(X, Wg, 1e-6), Y)
    e.emit_channelscale(X, Wg, Y, 9, 333)
    assert np.array_equal(O.channelscale_f32(X, Wg), Y)
