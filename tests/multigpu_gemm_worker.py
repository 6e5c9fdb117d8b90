"""Worker for tests/test_gpu_multi.py (launched by torchrun, one rank per GPU):
the N-sharded f16 GEMM with the fused all-gather must leave the same full C
on every rank as a single-GPU GEMM of the same inputs."""
import datetime
import os
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import unikern_b200.abi as abi  # noqa: E402
from unikern_b200 import shard  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", int(os.environ["LOCAL_RANK"])))
    ok = True
    for (M, N, K) in [(1024, 2048, 512), (384, 1000, 264), (8192, 8192, 1024)]:
        g = torch.Generator(device="cuda")
        g.manual_seed(M + N + K)
        A = (torch.randn((M, K), generator=g, device="cuda") * 0.5).half()
        B = (torch.randn((K, N), generator=g, device="cuda") * 0.5).half()
        C = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
        plan = shard.GemmAllGather(C, M, N, K)
        for _ in range(2):
            plan.run(A, plan.b_shard(B), C)
        ref = torch.empty_like(C)
        abi.gemm_f16(A, B, ref)
        torch.cuda.synchronize()
        diff = (C.float() - ref.float()).abs().max().item()
        fault = abi.lib().uk_cuda_pipeline_fault()
        print("rank %d %dx%dx%d max|C - single GPU| = %g fault=%d" % (rank, M, N, K, diff, fault), flush=True)
        ok = ok and diff == 0.0 and fault == 0
        dist.barrier()
        plan.close()
        del C
    dist.destroy_process_group()
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
