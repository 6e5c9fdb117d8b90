"""Multi-GPU parity: the N-sharded f16 GEMM with the all-gather fused into
its epilogue, on 2 GPUs (skipped where fewer GPUs are visible)."""
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu


def test_gemm_allgather_two_gpus_matches_single_gpu():
    import torch
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 GPUs, %d visible" % n)
    worker = Path(__file__).with_name("multigpu_gemm_worker.py")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29517", str(worker)]
    r = subprocess.run(cmd, capture_output=True, text=True, env={**__import__("os").environ, "NCCL_NVLS_ENABLE": "0"})
    print(r.stdout[-3000:], r.stderr[-3000:])
    assert r.returncode == 0
