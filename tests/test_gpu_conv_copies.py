"""The tensor-core fp32 conv writing several copies of its output
(uk_cuda_conv2d_f32_allgather), on one GPU with every copy local: the store
the batch-sharded multi-GPU conv uses for its fused all-gather.  Every copy
must hold exactly the one-copy result at this rank's images, nothing else."""
import ctypes as C

import numpy as np
import pytest

import unikern_b200.abi as abi
from oracle import oracle as O
from uk_testutil import F32_TOL, SUM_TAU, dev, host, torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("N_total,b0,b1,Cc,H,W,Oc,copies", [
    (8, 2, 4, 64, 28, 28, 64, 2),       # a middle block, two copies
    (32, 28, 32, 256, 56, 56, 256, 8),  # the 8-GPU shard of the BASELINE conv, eight copies
    (5, 0, 3, 32, 13, 11, 40, 3),       # ragged rows, channels past a tile
])
def test_conv_copies_match_one_copy(N_total, b0, b1, Cc, H, W, Oc, copies):
    t = torch()
    rng = np.random.default_rng(N_total * 100 + Cc + copies)
    x = rng.uniform(0, 1, (N_total, Cc, H, W)).astype(np.float32)
    w = rng.normal(0, np.sqrt(2.0 / (9 * Cc)), (Oc, Cc, 3, 3)).astype(np.float32)
    s = rng.uniform(0.5, 1.5, Oc).astype(np.float32)
    n = b1 - b0
    xd, wd, sd = dev(x[b0:b1]), dev(w), dev(s)
    one = t.empty((n, Oc, H, W), device="cuda")
    abi.conv2d_tc(xd, wd, one, n, H, W, Cc, 3, 3, Oc, 1, sd, abi.UK_CONV_NCHW)
    Ys = [t.full((N_total, Oc, H, W), -7.0, device="cuda") for _ in range(copies)]
    plane = Oc * H * W * 4
    ptrs = (C.c_void_p * copies)(*[y.data_ptr() + b0 * plane for y in Ys])
    ws = abi.conv2d_workspace(n, H, W, Cc, 3, 3, Oc, 1, abi.UK_CONV_NCHW)
    abi.check(abi.lib().uk_cuda_conv2d_f32_allgather(xd.data_ptr(), wd.data_ptr(), ptrs, copies, n, H, W, Cc, 3, 3,
                                                     Oc, 1, sd.data_ptr(), ws.data_ptr(),
                                                     ws.numel() * ws.element_size(), None))
    t.cuda.synchronize()
    assert abi.lib().uk_cuda_pipeline_fault() == 0
    want = host(one)
    for y in Ys:
        got = host(y)
        assert np.array_equal(got[b0:b1], want)
        assert (got[:b0] == -7.0).all() and (got[b1:] == -7.0).all()
    ref = O.conv_nchw(x[b0:b0 + 1], w, s, 1)
    assert O.rel_err(want[:1], ref, SUM_TAU * O.rms(ref)) <= F32_TOL
