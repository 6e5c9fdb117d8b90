"""The N-sharded GEMM from a C-ABI host over NCCL (uk_nccl_* /
uk_shard_gemm_f16_*), on 2 GPUs as child processes (skipped with fewer), with
NVLS off: parity of every rank's gathered C, and failure detection that ends
in code 4 (UK_ECUDA) within the limit -- a rank that never joins, and one
that stalls past the limit between steps.  No GPU is faulted, trapped or
hung: waits are bounded on the host, the communicator is aborted, and every
process lives until all have reported."""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
WORKER = Path(__file__).with_name("shard_nccl_worker.py")


def run(tmp_path, mode, world=2):
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip("needs %d GPUs, %d visible" % (world, torch.cuda.device_count()))
    env = {**os.environ, "NCCL_NVLS_ENABLE": "0"}
    procs = [subprocess.Popen(["timeout", "-k", "30", "300", sys.executable, str(WORKER), str(r), str(world),
                               str(tmp_path), mode], env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT,
                              text=True) for r in range(world)]
    logs = [p.communicate()[0] for p in procs]
    for p, log in zip(procs, logs):
        assert p.returncode == 0, log[-3000:]
    return [json.loads((tmp_path / ("result.%d.json" % r)).read_text()) for r in range(world)]


def test_sharded_gemm_from_the_c_abi_matches_the_oracle(tmp_path):
    for res in run(tmp_path, "ok"):
        assert res["init_rc"] == 0, res
        for e in res["shapes"]:
            assert all(s["rc"] == 0 for s in e["steps"]), e
            assert e["fault"] == 0
            assert e["max_diff_vs_one_gpu"] == 0.0
            assert e["err_vs_f64"] <= 2e-2


def test_a_rank_that_never_joins_ends_init_with_code_4(tmp_path):
    res = run(tmp_path, "never_joins")
    r0 = res[0]
    assert r0["init_rc"] == 4 and r0["init_s"] < 30, r0
    assert "did not arrive" in r0["init_err"] or "NCCL reported" in r0["init_err"], r0


def test_a_stalled_rank_ends_the_next_step_with_code_4(tmp_path):
    res = run(tmp_path, "stall")
    for r in res:
        steps = r["shapes"][0]["steps"]
        assert steps[0]["rc"] == 0, r
        assert len(steps) == 2 and steps[1]["rc"] == 4 and steps[1]["s"] < 30, r
        assert "communicator aborted" in steps[1]["err"], r
