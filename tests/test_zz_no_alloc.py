"""uk_cuda_reduce_f32_noalloc: the reduce for callers that cannot allocate
device memory (for example a plugin whose host application owns every device
allocation, or a caller that must not risk an allocation's synchronisation or
out-of-memory failure mid-run), so they have no workspace to pass.

Called through the C ABI and compared with the existing entry point
uk_cuda_reduce_f32 (given a workspace) on two calls in a row, within the f32
tolerance the other parity tests use.  The file name sorts last so that a
`-x` run has already run every other test if this one fails; it also passes
alone in a fresh process.
"""
import numpy as np
import pytest

import unikern_b200.abi as abi
from oracle import oracle as O
from uk_testutil import F32_TOL, SUM_TAU, dev, empty, host, torch

pytestmark = pytest.mark.gpu


def with_workspace(dX, rows, cols):
    t = torch()
    Y = empty((rows,))
    nbytes = abi.reduce_workspace_size(rows, cols)
    ws = t.empty(max(1, nbytes // 4), dtype=t.float32, device="cuda") if nbytes else None
    abi.check(abi.lib().uk_cuda_reduce_f32(dX.data_ptr(), Y.data_ptr(), rows, cols,
                                           ws.data_ptr() if ws is not None else None, nbytes,
                                           t.cuda.current_stream().cuda_stream))
    return host(Y)


def no_alloc(dX, rows, cols):
    t = torch()
    Y = empty((rows,))
    abi.check(abi.lib().uk_cuda_reduce_f32_noalloc(dX.data_ptr(), Y.data_ptr(), rows, cols,
                                                   t.cuda.current_stream().cuda_stream))
    return host(Y)


@pytest.mark.parametrize("rows,cols", [(1, 1 << 22), (3, 5000001), (17, 300000), (1, 134217728 // 8),
                                       (8192, 16384), (64, 100)])
def test_no_alloc_matches_workspace_entry_two_calls(rows, cols):
    for call in range(2):
        rng = np.random.default_rng(1000 * call + rows + cols)
        X = rng.normal(0, 1, (rows, cols)).astype(np.float32)
        dX = dev(X)
        want = with_workspace(dX, rows, cols)
        got = no_alloc(dX, rows, cols)
        tau = SUM_TAU * max(O.rms(want), np.sqrt(cols))
        assert O.rel_err(got, want, tau) <= F32_TOL
        # same kernels and the same plan: the bits agree as well
        assert np.array_equal(got, want)


def test_no_alloc_leaves_no_stale_partials():
    # a long call followed by a shorter one that uses fewer partial slots
    a = dev(np.full((1, 1 << 23), 0.5, np.float32))
    b = dev(np.full((1, 1 << 20), 0.015625, np.float32))
    assert no_alloc(a, 1, 1 << 23)[0] == float(1 << 22)
    assert no_alloc(b, 1, 1 << 20)[0] == 16384.0
    assert abi.lib().uk_cuda_pipeline_fault() == 0
