"""Multi-GPU parity on 2 GPUs (skipped where fewer GPUs are visible): the
N-sharded f16 GEMM with the all-gather fused into its epilogue, the
batch-sharded conv (NCCL all-gather of Y, or the gather fused into the conv's
store) and the weight-column-sharded decode.  Each runs with the ranks
ordered by the device-side flag barrier with the fused conv gather (the
default) and by a one-float NCCL all-reduce with the NCCL all-gather of the
conv (UK_BARRIER=nccl, UK_CONV_GATHER=nccl).  Each worker compares every rank's full output with a
single-GPU run of the same inputs and with the f64 oracle."""
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu


MODES = {"device": {}, "nccl": {"UK_BARRIER": "nccl", "UK_CONV_GATHER": "nccl"}}


def _torchrun(worker, port, mode="nccl"):
    import torch
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 GPUs, %d visible" % n)
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=%d" % port,
           str(Path(__file__).with_name(worker))]
    r = subprocess.run(cmd, capture_output=True, text=True,
                       env={**os.environ, "NCCL_NVLS_ENABLE": "0", **MODES[mode]})
    print(r.stdout[-3000:], r.stderr[-3000:])
    assert r.returncode == 0


@pytest.mark.parametrize("mode", list(MODES))
def test_gemm_allgather_two_gpus_matches_single_gpu(mode):
    _torchrun("multigpu_gemm_worker.py", 29517 + 10 * list(MODES).index(mode), mode)


@pytest.mark.parametrize("mode", list(MODES))
def test_conv_batch_shard_two_gpus_matches_single_gpu(mode):
    _torchrun("multigpu_conv_worker.py", 29518 + 10 * list(MODES).index(mode), mode)


@pytest.mark.parametrize("mode", list(MODES))
def test_decode_column_shard_two_gpus_matches_single_gpu(mode):
    _torchrun("multigpu_decode_worker.py", 29519 + 10 * list(MODES).index(mode), mode)
