"""Worker for tests/test_gpu_shard_nccl.py: one process per GPU, talking only
through the library's C ABI (uk_nccl_* / uk_shard_gemm_f16_*; torch is used
for device memory and the stream only).

    python shard_nccl_worker.py <rank> <world> <workdir> <mode>

mode ok          two steps of the N-sharded GEMM (8192^3 with BASELINE inputs,
                 and a ragged shape): every rank's full C against the fp64
                 oracle on sampled rows and bit for bit against one-GPU runs
mode stall       one step, then the last rank stops stepping for longer than
                 the others' limit: their next step must end with code 4
                 within about that limit, and so must the staller's
mode never_joins the last rank never creates its communicator: the others'
                 init must end with code 4 within the limit
Every process stays alive until all have written their result, so no NCCL
or library kernel ever reaches the memory of a process that has exited.
Writes <workdir>/result.<rank>.json.
"""
import ctypes as C
import json
import os
import sys
import time
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

import numpy as np  # noqa: E402
import torch  # noqa: E402

import unikern_b200.abi as abi  # noqa: E402
from oracle import oracle as O  # noqa: E402


def wait_for(path, limit_s):
    t0 = time.monotonic()
    while not path.exists():
        if time.monotonic() - t0 > limit_s:
            return False
        time.sleep(0.05)
    return True


def main():
    rank, world, work, mode = int(sys.argv[1]), int(sys.argv[2]), Path(sys.argv[3]), sys.argv[4]
    torch.cuda.set_device(rank)
    lib = abi.lib()
    res = {"rank": rank, "mode": mode}
    idfile = work / "nccl.id"
    if rank == 0:
        uid = C.create_string_buffer(lib.uk_nccl_unique_id_size())
        abi.check(lib.uk_nccl_get_unique_id(uid))
        tmp = work / "nccl.id.tmp"
        tmp.write_bytes(uid.raw)
        tmp.rename(idfile)
    assert wait_for(idfile, 60), "no NCCL id"
    uid = C.create_string_buffer(idfile.read_bytes(), lib.uk_nccl_unique_id_size())
    comm = C.c_void_p()
    limit_ns = int(3e9)
    staller = rank == world - 1

    if mode == "never_joins" and staller:
        res["rc"] = "did not join"
    else:
        t0 = time.monotonic()
        rc = lib.uk_nccl_comm_init(uid, world, rank, limit_ns if mode == "never_joins" else int(60e9), C.byref(comm))
        res["init_rc"], res["init_s"] = rc, time.monotonic() - t0
        res["init_err"] = lib.uk_cuda_last_error().decode() if rc else ""

    if mode in ("ok", "stall") and res.get("init_rc") == 0:
        stream = torch.cuda.current_stream()
        shapes = [(8192, 8192, 8192, 0.02), (300, 1000, 264, 0.5)] if mode == "ok" else [(1024, 2048, 512, 0.5)]
        res["shapes"] = []
        for (M, N, K, sd) in shapes:
            g = torch.Generator(device="cuda")
            g.manual_seed(M + N + K)
            A = (torch.randn((M, K), generator=g, device="cuda") * sd).half()
            B = (torch.randn((K, N), generator=g, device="cuda") * sd).half()
            Cm = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
            h = C.c_void_p()
            abi.check(lib.uk_shard_gemm_f16_create(comm, rank, world, Cm.data_ptr(), N, M, N, K, int(30e9),
                                                   C.byref(h)))
            n0, n1 = C.c_int64(), C.c_int64()
            abi.check(lib.uk_shard_gemm_f16_columns(h, C.byref(n0), C.byref(n1)))
            Bs = B[:, n0.value:n1.value].contiguous()
            steps = []
            for step in range(2):
                if mode == "stall" and step == 1 and staller:
                    time.sleep(8.0)  # stop stepping past the peers' 3 s limit
                t0 = time.monotonic()
                rc = lib.uk_shard_gemm_f16_run(h, A.data_ptr(), K, Bs.data_ptr(), n1.value - n0.value,
                                               stream.cuda_stream, limit_ns if mode == "stall" else int(30e9))
                steps.append({"rc": rc, "s": time.monotonic() - t0,
                              "err": lib.uk_cuda_last_error().decode() if rc else ""})
                if rc:
                    break
            entry = {"shape": [M, N, K], "steps": steps, "fault": lib.uk_cuda_pipeline_fault()}
            if mode == "ok" and all(s["rc"] == 0 for s in steps):
                torch.cuda.synchronize()
                ref = torch.empty_like(Cm)
                abi.gemm_f16(A, B, ref)
                torch.cuda.synchronize()
                entry["max_diff_vs_one_gpu"] = float((Cm.float() - ref.float()).abs().max().item())
                rows = np.unique(np.random.default_rng(rank).choice(M, min(M, 8), replace=False))
                Ah = A.cpu().view(torch.int16).numpy().view(np.uint16)
                Bh = B.cpu().view(torch.int16).numpy().view(np.uint16)
                f64 = O.gemm_f16_f64(Ah[rows], Bh, threads=O.nthreads())
                got = O.f16_to_f32(Cm.cpu().view(torch.int16).numpy().view(np.uint16)[rows])
                entry["err_vs_f64"] = O.rel_err(got, f64, O.rms(f64))
            lib.uk_shard_gemm_f16_destroy(h)
            res["shapes"].append(entry)
        torch.cuda.synchronize()
    if comm.value:
        lib.uk_nccl_comm_destroy(comm)
    out = work / ("result.%d.json" % rank)
    out.write_text(json.dumps(res))
    # stay alive until every rank has reported (no kernel of a live rank may
    # reach the memory of a process that already exited)
    for r in range(world):
        wait_for(work / ("result.%d.json" % r), 60)
    return 0


if __name__ == "__main__":
    sys.exit(main())
