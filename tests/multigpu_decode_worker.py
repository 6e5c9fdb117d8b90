"""Worker for tests/test_gpu_multi.py (launched by torchrun, one rank per GPU):
the decode layer with its weight columns sharded over the ranks and the
all-gather fused into the GEMM's store must leave on every rank the full
Y[B][N] of a single-GPU run (up to f16 rounding: the K split of a narrow
shard sums in a different order), and that Y must agree on every rank with
the fp64 oracle of the op-by-op chain (the reference's fp32 RMSNorm rounded to
f16, then the product in fp64) within the f16 GEMM gate."""
import datetime
import os
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import numpy as np  # noqa: E402

import unikern_b200.abi as abi  # noqa: E402
from oracle import oracle as O  # noqa: E402
from unikern_b200 import shard  # noqa: E402


def main():
    rank = int(os.environ["RANK"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", int(os.environ["LOCAL_RANK"])))
    ok = True
    for (B, K, N) in [(32, 4096, 14336), (3, 1024, 1000)]:
        g = torch.Generator(device="cuda")
        g.manual_seed(B + K + N)
        X = torch.randn((B, K), generator=g, device="cuda")
        gamma = torch.randn((K,), generator=g, device="cuda") * 0.1 + 1.0
        W = (torch.randn((K, N), generator=g, device="cuda") * 0.02).half()
        Y = torch.full((B, N), float("nan"), dtype=torch.float16, device="cuda")
        plan = shard.DecodeColumnShard(Y, B, N, K)
        Ws = plan.w_shard(W)
        for _ in range(2):
            plan.run(X, gamma, Ws)
        ref = torch.empty_like(Y)
        abi.decode_rmsnorm_gemm(X, gamma, W, ref, 1e-5)
        torch.cuda.synchronize()
        diff = (Y.float() - ref.float()).abs().max().item()
        scale = ref.float().abs().max().item()
        fault = abi.lib().uk_cuda_pipeline_fault()
        print("rank %d decode %dx%dx%d max|Y - single GPU| = %g (of %g) fault=%d" % (rank, B, K, N, diff, scale,
                                                                                   fault), flush=True)
        ok = ok and diff <= 2e-3 * scale and fault == 0 and not torch.isnan(Y.float()).any().item()
        Wh = W.cpu().view(torch.int16).numpy().view(np.uint16)
        ref = O.gemm_f16_f64(O.f32_to_f16(O.rmsnorm_f32(X.cpu().numpy(), gamma.cpu().numpy(), 1e-5)), Wh,
                             threads=O.nthreads())
        got = O.f16_to_f32(Y.cpu().view(torch.int16).numpy().view(np.uint16))
        err = O.rel_err(got, ref, O.rms(ref))
        print("rank %d decode %dx%dx%d full Y vs f64: %.3e" % (rank, B, K, N, err), flush=True)
        ok = ok and err <= 2e-2
        dist.barrier()
        plan.close()
        del Y
    dist.destroy_process_group()
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
