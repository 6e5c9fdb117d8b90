"""The f16 GEMM writing several copies of C (uk_cuda_gemm_f16_allgather), on
one GPU with every copy local: the epilogues that the N-sharded multi-GPU
GEMM uses for its fused all-gather (lane stores to every copy, and the
opt-in TMA tensor stores of each staged 32 x 64 block, in a child process
with UNIKERN_GEMM_F16_TMA_OUT=1).  Each copy must hold exactly the one-copy
result, only in this rank's columns, with the ragged edges of M and N
clipped and nothing written outside the block."""
import ctypes as C

import numpy as np
import pytest

import unikern_b200.abi as abi
from oracle import oracle as O
from uk_testutil import F16_TOL, SUM_TAU, dev, host, torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N_total,col0,ncols,K,copies", [
    (1024, 2048, 512, 1024, 512, 2),     # an even shard, two copies
    (8192, 8192, 1024, 1024, 1024, 8),   # the 8-GPU shard shape, eight copies
    (300, 1000, 200, 424, 264, 3),       # ragged: 300 rows (box rows clipped), 424 columns (box columns clipped)
    (130, 520, 8, 136, 64, 4),           # a single pair row of tiles, narrow shard
])
def test_copies_match_one_copy(M, N_total, col0, ncols, K, copies):
    t = torch()
    rng = np.random.default_rng(M + ncols + copies)
    Ah = O.f32_to_f16(rng.normal(0, 0.5, (M, K)).astype(np.float32))
    Bh = O.f32_to_f16(rng.normal(0, 0.5, (K, N_total)).astype(np.float32))
    A, B = dev(Ah), dev(Bh)
    Bs = B[:, col0:col0 + ncols]
    # reference: the one-copy GEMM of the same column block
    one = t.empty((M, ncols), dtype=t.float16, device="cuda")
    abi.gemm_f16(A, Bs.contiguous(), one)
    sentinel = t.tensor(-7.0, dtype=t.float16)
    Cs = [t.full((M, N_total), -7.0, dtype=t.float16, device="cuda") for _ in range(copies)]
    ptrs = (C.c_void_p * copies)(*[c.data_ptr() for c in Cs])
    abi.check(abi.lib().uk_cuda_gemm_f16_allgather(A.data_ptr(), K, Bs.data_ptr(), N_total, ptrs, copies, N_total,
                                                   M, ncols, K, col0, t.cuda.current_stream().cuda_stream))
    t.cuda.synchronize()
    assert abi.lib().uk_cuda_pipeline_fault() == 0
    want = host(one)
    for c in Cs:
        got = host(c)
        assert np.array_equal(got[:, col0:col0 + ncols], want)
        outside = np.concatenate([got[:, :col0].reshape(-1), got[:, col0 + ncols:].reshape(-1)])
        assert (outside == host(sentinel.cuda().reshape(1))[0]).all(), "a copy was written outside its block"
    # and the block is right (rows sampled against f64)
    rows = [0, M // 2, M - 1]
    ref = O.gemm_f16_f64(Ah[rows], Bh[:, col0:col0 + ncols], threads=8)
    assert O.rel_err(O.f16_to_f32(want[rows]), ref, SUM_TAU * O.rms(ref)) <= F16_TOL


def test_tma_store_epilogue_in_a_child_process():
    # the epilogue choice is read once per process: run the same cases with
    # the TMA-store epilogue in a fresh one
    import os
    import subprocess
    import sys
    from pathlib import Path
    here = Path(__file__).resolve().parent
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", str(here / "test_gpu_gemm_copies.py"), "-m", "gpu",
                        "-k", "test_copies_match_one_copy"], capture_output=True, text=True, timeout=600,
                       env={**os.environ, "UNIKERN_GEMM_F16_TMA_OUT": "1"})
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
