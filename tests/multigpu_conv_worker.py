"""Worker for tests/test_gpu_multi.py (launched by torchrun, one rank per GPU):
the batch-sharded conv with the NCCL all-gather of Y must leave on every rank
the same full Y, bit for bit, as a single-GPU run of the same kernel over the
whole batch (to the fp32 gate: see below), and images of every rank's shard
must agree with the fp64 oracle of the reference's cpu_conv
(src/reference.cpp:6-22) on every rank."""
import datetime
import os
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import unikern_b200.abi as abi  # noqa: E402
from oracle import oracle as O  # noqa: E402
from unikern_b200 import shard  # noqa: E402


def main():
    rank = int(os.environ["RANK"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", int(os.environ["LOCAL_RANK"])))
    ok = True
    for (N, Cc, H, W, Oc, pad) in [(32, 64, 28, 28, 64, 1), (5, 16, 13, 11, 24, 1), (8, 256, 56, 56, 256, 1)]:
        g = torch.Generator(device="cuda")
        g.manual_seed(N * 1000 + Cc)
        x = torch.rand((N, Cc, H, W), generator=g, device="cuda")
        w = torch.randn((Oc, Cc, 3, 3), generator=g, device="cuda") * (2.0 / (9 * Cc)) ** 0.5
        s = torch.rand((Oc,), generator=g, device="cuda") + 0.5
        plan = shard.ConvBatchShard(N, Cc, H, W, Oc, 3, 3, pad)
        Y = torch.full((N, Oc, plan.Ho, plan.Wo), float("nan"), device="cuda")
        plan.run(plan.x_shard(x).contiguous(), w, Y, s)
        ref = torch.empty_like(Y)
        abi.conv2d_tc(x, w, ref, N, H, W, Cc, 3, 3, Oc, pad, s, abi.UK_CONV_NCHW)  # same kernel, one GPU
        torch.cuda.synchronize()
        diff = (Y - ref).abs().max().item()
        rel = diff / ref.abs().max().item()
        print("rank %d conv N=%d C=%d %dx%d -> %d: max|Y - single GPU| = %g (rel %g)" % (rank, N, Cc, H, W, Oc, diff,
                                                                                         rel), flush=True)
        # every image runs the same tiles with the same k-order on either GPU
        # count, except the last round of tiles, which is split along K by the
        # tile count: a different grouping in the tensor cores' accumulator
        # there (~2e-5 of the output scale), so the fp32 gate, not bitwise
        ok = ok and rel <= 1e-4 and not torch.isnan(Y).any().item()
        print("rank %d conv gather: %s" % (rank, plan.describe()), flush=True)
        # the first and last image (different ranks' shards) against fp64
        xs, ws_, ss = x.cpu().numpy(), w.cpu().numpy(), s.cpu().numpy()
        Yh = Y.cpu().numpy()
        for n in sorted({0, N - 1}):
            ref_n = O.conv_nchw(xs[n:n + 1], ws_, ss, pad)
            err = O.rel_err(Yh[n:n + 1], ref_n, O.rms(ref_n))
            print("rank %d conv image %d vs f64: %.3e" % (rank, n, err), flush=True)
            ok = ok and err <= 1e-4
        dist.barrier()
        plan.close()
    dist.destroy_process_group()
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
