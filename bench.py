#!/usr/bin/env python
"""bench.py -- throughput of the B200 KML operator set (one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--op OP]

Headline workload (``value``): f16 GEMM, C(f16) = A(f16) * B(f16) with f32
accumulation, M = N = K = 8192 row-major; at N GPUs
the columns of B and C are split over the ranks (strong scaling, total work
fixed).  A step is one GEMM over inputs already resident in HBM; ``e2e`` is
the same metric through the C ABI with pinned host buffers copied in and the
result copied out inside the timed region.

The line also carries ``ops``: the other KML ops at their BASELINE sizes on
rank 0 (row reduce / RMSNorm / softmax over [8192 x 16384], channelscale,
the KML scalar reduce, the conv N=32 256->256 56x56 3x3 pad 1 with the fused
channel scale, the f32 GEMM 512^3 and the decode chain), each with its own
roofline and a CPU baseline on a bounded sample.

Timing: W untimed steps, then exactly K steps between CUDA events on the
launching stream, barrier + synchronize on both sides, max over ranks.
Inputs are larger than L2 (126 MB) for every HBM-bound op and the GEMM.
``--impl reference`` times the reference's own CPU implementation of the
headline op on all host cores (rank 0; other ranks exit 0).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = json.loads((ROOT / "BASELINE.json").read_text())["metric"] if (ROOT / "BASELINE.json").exists() else \
    "f16 GEMM TFLOP/s; reduce/norm/softmax HBM GB/s; % roofline at 1/2/4/8 B200"
FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
FP32_SIMT_TFLOPS = 2 * 148 * 128 * 1.965e9 / 1e12  # nominal FFMA peak (no measured figure exists)


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        d["source"] = "measured"
        return d
    d = dict(FALLBACK)
    d["source"] = "fallback"
    return d


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.file = None

    def start(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.idx), "--query-gpu=" + self.FIELDS,
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.file, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.05)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        rows = []
        for line in Path(self.file.name).read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) >= 9:
                rows.append(f)
        os.unlink(self.file.name)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------
# timing
# ---------------------------------------------------------------------------
class Ctx:
    def __init__(self, world, rank, local_rank):
        import torch
        self.torch = torch
        self.world, self.rank, self.local_rank = world, rank, local_rank
        self.stream = torch.cuda.current_stream()

    def barrier(self):
        if self.world > 1:
            self.torch.distributed.barrier()

    def max_over_ranks(self, v):
        if self.world == 1:
            return v
        t = self.torch.tensor([v], dtype=self.torch.float64, device="cuda")
        self.torch.distributed.all_reduce(t, op=self.torch.distributed.ReduceOp.MAX)
        return float(t.item())

    def time_steps(self, step, steps, warmup, flush=None):
        """ms per step over exactly `steps` launches (events on the launching stream)."""
        torch = self.torch
        for _ in range(warmup):
            step()
        torch.cuda.synchronize()
        self.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(self.stream)
        for _ in range(steps):
            step()
        e1.record(self.stream)
        torch.cuda.synchronize()
        self.barrier()
        torch.cuda.synchronize()
        return self.max_over_ranks(e0.elapsed_time(e1) / steps)


# ---------------------------------------------------------------------------
# CPU baselines (the reference's own CPU code where oracle/_ref was built,
# else the oracle port; both are the checker, timed here only)
# ---------------------------------------------------------------------------
def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def run_threads(fn, n):
    ths = [threading.Thread(target=fn, args=(i,)) for i in range(n)]
    t0 = time.perf_counter()
    for t in ths:
        t.start()
    for t in ths:
        t.join()
    return time.perf_counter() - t0


def cpu_gemm_f16(M, N, K, budget_s=10.0, rows=None):
    """Rows of C = A * B (8192^3 f16 config) with the reference's cpu_ref loop
    (src/codegen_hip.cpp:1124-1132 on half-quantised inputs); one row per thread."""
    import numpy as np
    from oracle import oracle as O
    nt = cpu_threads()
    rng = np.random.default_rng(5)
    Bh = O.f32_to_f16(rng.normal(0, 0.02, (K, N)).astype(np.float32))
    e = O.emit()
    kind = "reference" if e is not None else "port"
    nrows = rows or nt
    Ah = O.f32_to_f16(rng.normal(0, 0.02, (nrows, K)).astype(np.float32))
    if e is not None:
        Bf = O.f16_to_f32(Bh)
        e.emit_gemm_set_B(Bf, K, N)
        Af = O.f16_to_f32(Ah)
        out = np.zeros((nrows, N), np.float32)

        def work(t):  # thread t takes rows t, t + nt, ...
            for i in range(t, nrows, nt):
                e.emit_gemm_f16_rows(Af[i:i + 1].copy(), out[i:i + 1], 1)
        dt = run_threads(work, min(nt, nrows))
    else:
        t0 = time.perf_counter()
        O.gemm_f16(np.vstack([Ah, np.zeros((0, K), np.uint16)]), Bh, rows=(0, nrows), threads=nt)
        dt = time.perf_counter() - t0
    flops = 2.0 * nrows * N * K
    return {"value": flops / dt / 1e12, "unit": "TFLOP/s", "cores": min(nt, nrows), "kind": kind,
            "sample": "%d rows x %d cols of C (K=%d), %.2f s, extrapolated to the full %dx%dx%d GEMM by rate"
                      % (nrows, N, K, dt, M, N, K), "seconds": dt}


def cpu_rowop(op, L, C, budget_rows=None):
    import numpy as np
    from oracle import oracle as O
    nt = cpu_threads()
    rows = budget_rows or L  # the whole workload: it takes well under a minute on the host
    rng = np.random.default_rng(6)
    X = rng.normal(0, 1, (rows, C)).astype(np.float32)
    W = rng.normal(1, 0.1, C).astype(np.float32)
    e, r = O.emit(), O.ref()
    kind = "reference" if (e is not None and r is not None) else "port"
    per = (rows + nt - 1) // nt
    out = np.zeros_like(X)
    ysum = np.zeros(rows, np.float32)

    def work(i):
        a, b = i * per, min(rows, (i + 1) * per)
        if a >= b:
            return
        xs = np.ascontiguousarray(X[a:b])
        if kind == "reference":
            if op == "softmax":
                e.emit_softmax(xs, out[a:b], b - a, C)
            elif op == "rmsnorm":
                e.emit_rmsnorm(xs, W, out[a:b], b - a, C)
            elif op == "channelscale":
                e.emit_channelscale(xs, W, out[a:b], b - a, C)
            else:
                for j in range(a, b):
                    ysum[j] = r.ref_cpu_reduce_blocked(X[j], C, 1024)
        else:
            if op == "softmax":
                O.lib().or_softmax_f32(xs, out[a:b], b - a, C, 1)
            elif op == "rmsnorm":
                O.lib().or_rmsnorm_f32(xs, W, out[a:b], b - a, C, 1e-6, 1)
            elif op == "channelscale":
                O.lib().or_channelscale_f32(xs, W, out[a:b], b - a, C, 1)
            else:
                O.lib().or_row_reduce_f32(xs, ysum[a:b], b - a, C, 1024, 1)
    dt = run_threads(work, nt)
    nbytes = rows * C * 4 * (1 if op == "reduce" else 2)
    return {"value": nbytes / dt / 1e9, "unit": "GB/s", "cores": nt, "kind": kind,
            "sample": "%d of %d rows (C=%d, one contiguous block of rows per thread), %.2f s%s" % (rows, L, C, dt,
                                                           "; eps fixed at 1e-6 in the reference" if op == "rmsnorm" else ""),
            "seconds": dt}


def cpu_conv(N, Cc, H, W, Oc, pad):
    """The reference's cpu_conv (src/reference.cpp:6-22) on host-padded HWC
    images, one image per thread; extrapolated to N images by rate."""
    import numpy as np
    from oracle import oracle as O
    r = O.ref()
    nt = min(cpu_threads(), N)
    Hp, Wp = H + 2 * pad, W + 2 * pad
    rng = np.random.default_rng(7)
    x = rng.uniform(0, 1, (Hp, Wp, Cc)).astype(np.float32).reshape(-1)
    w = rng.normal(0, 0.03, (Oc, 3, 3, Cc)).astype(np.float32).reshape(-1)
    ys = [np.zeros(Oc * H * W, np.float32) for _ in range(nt)]

    def work(i):
        if r is not None:
            r.ref_cpu_conv(x, w, ys[i], Hp, Wp, Cc, 3, 3, Oc)
        else:
            O.lib().or_conv_f32(x, w, ys[i], Hp, Wp, Cc, 3, 3, Oc, 1)
    dt = run_threads(work, nt)
    flops = 2.0 * nt * H * W * Cc * 9 * Oc
    return {"value": flops / dt / 1e12, "unit": "TFLOP/s", "cores": nt, "kind": "reference" if r else "port",
            "sample": "%d images of %d (one per thread), %.2f s" % (nt, N, dt), "seconds": dt}


def cpu_gemm_f32(M=512, N=512, K=512):
    """The whole f32 GEMM with the reference's cpu_ref
    loop (src/codegen_hip.cpp:1124-1132), rows split over the host threads."""
    import numpy as np
    from oracle import oracle as O
    nt = cpu_threads()
    rng = np.random.default_rng(11)
    A = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    B = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    out = np.zeros((M, N), np.float32)
    e = O.emit()
    per = (M + nt - 1) // nt
    if e is not None:
        e.emit_gemm_set_B(B, K, N)

        def work(i):
            a, b = i * per, min(M, (i + 1) * per)
            if a < b:
                e.emit_gemm_rows(np.ascontiguousarray(A[a:b]), out[a:b], b - a)
        dt = run_threads(work, nt)
    else:
        t0 = time.perf_counter()
        O.gemm_f32(A, B, threads=nt)
        dt = time.perf_counter() - t0
    return {"value": 2.0 * M * N * K / dt / 1e12, "unit": "TFLOP/s", "cores": nt,
            "kind": "reference" if e is not None else "port",
            "sample": "the whole %dx%dx%d GEMM, rows split over %d threads, %.3f s" % (M, N, K, nt, dt), "seconds": dt}


def cpu_reduce_scalar(L=134217728):
    """The KML reduce (one vector of L floats to a scalar) with the reference's
    cpu_reduce_blocked (src/reference.cpp:36-48): one pass, one thread, as the
    reference runs it."""
    import numpy as np
    from oracle import oracle as O
    rng = np.random.default_rng(17)
    X = rng.normal(0, 1, L).astype(np.float32)
    r = O.ref()
    t0 = time.perf_counter()
    if r is not None:
        r.ref_cpu_reduce_blocked(X, L, 1024)
    else:
        O.reduce_blocked_f32(X, 1024)
    dt = time.perf_counter() - t0
    return {"value": L * 4 / dt / 1e9, "unit": "GB/s", "cores": 1, "kind": "reference" if r is not None else "port",
            "sample": "the whole vector (L = %d), %.3f s" % (L, dt), "seconds": dt}


def cpu_decode(Bt=32, H=4096, F=14336, heads=32, S=8192):
    """The decode chain on the host with the reference's CPU paths: cpu_rmsnorm
    (eps fixed at 1e-6 in the reference), the half-quantised f16 cpu_ref over
    the 32 token rows, cpu_softmax over the 1024 score rows; threads over rows."""
    import numpy as np
    from oracle import oracle as O
    e = O.emit()
    nt = cpu_threads()
    rng = np.random.default_rng(18)
    x = rng.normal(0, 1, (Bt, H)).astype(np.float32)
    g = rng.normal(1, 0.1, H).astype(np.float32)
    W = O.f16_to_f32(O.f32_to_f16(rng.normal(0, 0.02, (H, F)).astype(np.float32)))
    sc = rng.normal(0, 1, (Bt * heads, S)).astype(np.float32)
    xn = np.zeros_like(x)
    y = np.zeros((Bt, F), np.float32)
    pr = np.zeros_like(sc)
    if e is None:
        return None
    e.emit_gemm_set_B(W, H, F)
    sp = (Bt * heads + nt - 1) // nt

    def work(i):
        if i < Bt:
            e.emit_gemm_f16_rows(np.ascontiguousarray(xn[i:i + 1]), y[i:i + 1], 1)
        a, b = i * sp, min(Bt * heads, (i + 1) * sp)
        if a < b:
            e.emit_softmax(np.ascontiguousarray(sc[a:b]), pr[a:b], b - a, S)
    t0 = time.perf_counter()
    e.emit_rmsnorm(x, g, xn, Bt, H)
    run_threads(work, max(nt, 1))
    dt = time.perf_counter() - t0
    nbytes = Bt * H * 4 + H * 4 + H * F * 2 + Bt * F * 2 + 2 * Bt * heads * S * 4
    return {"value": nbytes / dt / 1e9, "unit": "GB/s", "cores": nt, "kind": "reference",
            "sample": "the whole chain (B = %d), %.3f s" % (Bt, dt), "seconds": dt}


def strip(d):
    return None if d is None else {k: (round(v, 6) if isinstance(v, float) else v) for k, v in d.items()
                                   if k != "seconds"}


# ---------------------------------------------------------------------------
# GPU workloads
# ---------------------------------------------------------------------------
def gen(torch, shape, kind, seed, dtype=None, scale=1.0, lo=0.0, hi=1.0):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    if kind == "normal":
        t = torch.randn(shape, generator=g, device="cuda") * scale
    else:
        t = torch.rand(shape, generator=g, device="cuda") * (hi - lo) + lo
    return t.to(dtype) if dtype is not None else t


def bench_gemm_f16(ctx, steps, warmup, M=8192, N=8192, K=8192):
    import unikern_b200.abi as abi
    torch = ctx.torch
    world, rank = ctx.world, ctx.rank
    A = gen(torch, (M, K), "normal", 1, torch.float16, 0.02)
    B = gen(torch, (K, N), "normal", 2, torch.float16, 0.02)
    Cm = torch.empty((M, N), dtype=torch.float16, device="cuda")
    if world == 1:
        def step():
            abi.gemm_f16(A, B, Cm)
        launches_per_step = 1
        parallelism = "single GPU"
        Bs = B
    else:
        from unikern_b200 import shard
        plan = shard.GemmAllGather(Cm, M, N, K)
        Bs = plan.b_shard(B)
        kev = []  # (start, end) events around this rank's GEMM launch in each timed step

        def step():
            if timing[0]:
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(ctx.stream)
                plan.launch(A, Bs)
                e1.record(ctx.stream)
                kev.append((e0, e1))
            else:
                plan.launch(A, Bs)
            plan.barrier()
        launches_per_step = plan.launches_per_step
        parallelism = plan.describe()
    timing = [False]
    for _ in range(warmup):
        step()
    timing[0] = True
    ms = ctx.time_steps(step, steps, 0)
    timing[0] = False
    flops = 2.0 * M * N * K
    if world == 1:
        kernel_ms, flops_per_launch = ms, flops
    else:
        # the dominant kernel's own launch time: events on the launching stream
        # around each GEMM (the barrier is outside), max over ranks
        kernel_ms = ctx.max_over_ranks(sum(a.elapsed_time(b) for a, b in kev) / len(kev))
        flops_per_launch = 2.0 * M * (plan.n1 - plan.n0) * K
    res = {"ms": ms, "value": flops / ms / 1e9, "flops_per_step": flops, "launches": launches_per_step * steps,
           "parallelism": parallelism, "kernel_ms": kernel_ms,
           "kernel_tflops": flops_per_launch / kernel_ms / 1e9}
    # e2e through the C ABI with pinned host buffers (rank-local inputs): on
    # one GPU the pipelined host-to-host entry point (uploads of A row blocks,
    # their GEMMs and the downloads of C blocks overlapped); on N GPUs each
    # rank uploads A and its B block, runs the sharded GEMM and downloads C
    Ah = A.cpu().pin_memory()
    Bh = Bs.contiguous().cpu().pin_memory()
    Ch = torch.empty((M, N), dtype=torch.float16).pin_memory()
    Bd = torch.empty_like(Bh, device="cuda")

    def e2e_step():
        if world == 1:
            abi.gemm_f16_host(Ah, Bh, Ch, A, Bd, Cm)
            return
        A.copy_(Ah, non_blocking=True)
        Bd.copy_(Bh, non_blocking=True)
        plan.run(A, Bd, Cm)
        Ch.copy_(Cm, non_blocking=True)
    e2e_ms = ctx.time_steps(e2e_step, max(2, min(steps, 10)), 1)
    if world > 1:
        # every rank must hold the same full C: spot-check against a column
        # block computed locally on this GPU
        ref = torch.empty((M, 64), dtype=torch.float16, device="cuda")
        j0 = ((rank + 1) % world) * (N // world)
        abi.gemm_f16(A, B[:, j0:j0 + 64], ref)
        step()
        torch.cuda.synchronize()
        res["allgather_max_abs_diff"] = float((Cm[:, j0:j0 + 64].float() - ref.float()).abs().max().item())
        plan.close()
    res["e2e"] = {"value": flops / e2e_ms / 1e9, "unit": "TFLOP/s",
                  "h2d_bytes_per_step": Ah.numel() * 2 + Bh.numel() * 2, "d2h_bytes_per_step": Ch.numel() * 2,
                  "ms_per_step": e2e_ms}
    return res


def bench_rowop(ctx, op, steps, warmup, L=8192, C=16384):
    import unikern_b200.abi as abi
    torch = ctx.torch
    X = gen(torch, (L, C), "normal", 3, None, 2.0 if op == "softmax" else 1.0)
    W = gen(torch, (C,), "normal", 4, None, 0.1) + 1.0
    Y = torch.empty((L, C), device="cuda")
    R = torch.empty((L,), device="cuda")
    if op == "rmsnorm":
        step = lambda: abi.rmsnorm(X, W, Y, 1e-5)  # noqa: E731
        nbytes = 2 * L * C * 4 + C * 4
    elif op == "softmax":
        step = lambda: abi.softmax(X, Y)  # noqa: E731
        nbytes = 2 * L * C * 4
    elif op == "channelscale":
        step = lambda: abi.channelscale(X, W, Y)  # noqa: E731
        nbytes = 2 * L * C * 4 + C * 4
    elif op == "reduce":
        step = lambda: abi.reduce(X, R)  # noqa: E731
        nbytes = L * C * 4 + L * 4
    elif op == "reduce_scalar":
        Xs = X.view(1, L * C)
        ws = torch.empty(max(1, abi.reduce_workspace_size(1, L * C) // 4), device="cuda")
        step = lambda: abi.reduce(Xs, R[:1], ws)  # noqa: E731
        nbytes = L * C * 4 + 4
    ms = ctx.time_steps(step, steps, warmup)
    return {"ms": ms, "value": nbytes / ms / 1e6, "bytes_per_step": nbytes}


def bench_conv(ctx, steps, warmup, N=32, Cc=256, H=56, W=56, Oc=256, pad=1):
    import unikern_b200.abi as abi
    torch = ctx.torch
    x = gen(torch, (N, Cc, H, W), "uniform", 8)
    w = gen(torch, (Oc, Cc, 3, 3), "normal", 9, None, (2.0 / (9 * Cc)) ** 0.5)
    s = gen(torch, (Oc,), "uniform", 10, None, lo=0.5, hi=1.5)
    y = torch.empty((N, Oc, H, W), device="cuda")
    ws = abi.conv2d_workspace(N, H, W, Cc, 3, 3, Oc, pad, abi.UK_CONV_NCHW)
    step = lambda: abi.conv2d_tc(x, w, y, N, H, W, Cc, 3, 3, Oc, pad, s, abi.UK_CONV_NCHW, ws)  # noqa: E731
    ms = ctx.time_steps(step, steps, warmup)
    flops = 2.0 * N * H * W * Cc * 9 * Oc
    return {"ms": ms, "value": flops / ms / 1e9, "flops_per_step": flops}


def bench_gemm_f32(ctx, steps, warmup, M=512, N=512, K=512):
    import unikern_b200.abi as abi
    torch = ctx.torch
    A = gen(torch, (M, K), "uniform", 11, lo=-1, hi=1)
    B = gen(torch, (K, N), "uniform", 12, lo=-1, hi=1)
    Cm = torch.empty((M, N), device="cuda")
    # a 512^3 GEMM is a few microseconds of device time: the step replays a
    # CUDA graph of the one launch so host launch overhead stays out
    graph = capture(ctx, lambda: abi.gemm_f32(A, B, Cm))
    ms = ctx.time_steps(graph.replay, steps, warmup)
    return {"ms": ms, "value": 2.0 * M * N * K / ms / 1e9, "graph": True}


def bench_gemm_f32_tc(ctx, steps, warmup, M=8192, N=8192, K=8192):
    """fp32 GEMM on the tensor cores (split-tf32 through the convolution's
    pair kernel); the step includes both tf32 pre-passes."""
    import unikern_b200.abi as abi
    torch = ctx.torch
    A = gen(torch, (M, K), "uniform", 11, lo=-1, hi=1)
    B = gen(torch, (K, N), "uniform", 12, lo=-1, hi=1)
    Cm = torch.empty((M, N), device="cuda")
    ws = abi.gemm_f32_workspace(M, N, K)
    ms = ctx.time_steps(lambda: abi.gemm_f32_tc(A, B, Cm, ws, ctx.stream), steps, warmup)
    return {"ms": ms, "value": 2.0 * M * N * K / ms / 1e9}


def bench_decode(ctx, steps, warmup, Bt=32, H=4096, F=14336, heads=32, S=8192):
    """Decode-layer chain: RMSNorm [B x 4096] fused into
    the f16 skinny GEMM [B x 4096] x [4096 x 14336] (one kernel), then softmax
    over [B*32 x 8192] scores.  HBM-bound: the 112 MiB of weights dominate."""
    import unikern_b200.abi as abi
    torch = ctx.torch
    x = gen(torch, (Bt, H), "normal", 13)
    g = gen(torch, (H,), "normal", 14, None, 0.1) + 1.0
    Wt = gen(torch, (H, F), "normal", 15, torch.float16, 0.02)
    out = torch.empty((Bt, F), dtype=torch.float16, device="cuda")
    sc = gen(torch, (Bt * heads, S), "normal", 16)
    pr = torch.empty_like(sc)

    ws = abi.decode_workspace(Bt, H)
    side = torch.cuda.Stream()

    def chain():
        # the softmax does not depend on the GEMM: it runs on a forked stream,
        # so the graph holds two branches and the softmax's CTAs use the SMs
        # the GEMM leaves free (112 of 148 stream the weight)
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            abi.softmax(sc, pr)
        abi.decode_rmsnorm_gemm(x, g, Wt, out, 1e-5, ws)
        torch.cuda.current_stream().wait_stream(side)
    # a decode step is a handful of short launches: it runs as one CUDA graph
    # (captured once, replayed every step) so host launch overhead stays out
    graph = capture(ctx, chain)
    ms = ctx.time_steps(graph.replay, steps, warmup)
    nbytes = Bt * H * 4 + H * 4 + H * F * 2 + Bt * F * 2 + 2 * Bt * heads * S * 4
    return {"ms": ms, "value": nbytes / ms / 1e6, "bytes_per_step": nbytes, "batch": Bt, "graph": True}


def bench_gemm_streamed(ctx, steps, warmup, M=32768, N=32768, K=32768, f16=False, block_rows=4096):
    """Scenario B (src/codegen_hip.cpp:1485-1500): C = A * B from and to
    page-locked host memory with only B resident and A / C streamed through a
    two-slot device ring of block_rows-row blocks.  Each step is the whole
    call: B's upload, every block's upload / GEMM / download, overlapped.
    32768^3 fp32 is the reference's published streamed run."""
    import unikern_b200.abi as abi
    torch = ctx.torch
    dt = torch.float16 if f16 else torch.float32
    Ah = torch.empty((M, K), dtype=dt, pin_memory=True)
    Bh = torch.empty((K, N), dtype=dt, pin_memory=True)
    Ch = torch.empty((M, N), dtype=dt, pin_memory=True)
    for h, seed in ((Ah, 21), (Bh, 22)):  # seeded uniform[-1, 1] rows, made on the device a block at a time
        g = torch.Generator(device="cuda")
        g.manual_seed(seed)
        for r0 in range(0, h.shape[0], 4096):
            blk = torch.rand((min(4096, h.shape[0] - r0), h.shape[1]), generator=g, device="cuda") * 2 - 1
            h[r0:r0 + blk.shape[0]].copy_(blk.to(dt))
    Bd = torch.empty((K, N), dtype=dt, device="cuda")
    ring = torch.empty(abi.lib().uk_cuda_gemm_streamed_ring_size(M, N, K, int(f16), block_rows), dtype=torch.uint8,
                       device="cuda")
    ms = ctx.time_steps(lambda: abi.gemm_streamed(Ah, Bh, Ch, Bd, ring, block_rows, ctx.stream), steps, warmup)
    es = 2 if f16 else 4
    host_bytes = (M * K + K * N + M * N) * es
    return {"ms": ms, "value": 2.0 * M * N * K / ms / 1e9, "link_GBps": host_bytes / ms / 1e6,
            "host_bytes": host_bytes, "blocks": (M + block_rows - 1) // block_rows}


def capture(ctx, fn):
    """fn's launches as a CUDA graph on the bench stream (after two eager
    warm-up calls that set up per-device state)."""
    torch = ctx.torch
    fn()
    fn()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):  # captured on a side stream, replayed on the bench stream
        fn()
    torch.cuda.synchronize()
    return graph


def bench_rowop_f16(ctx, op, steps, warmup, L=8192, C=16384):
    """The fp16 row ops (f16 rows in and out, fp32 arithmetic) at the BASELINE row shape."""
    import unikern_b200.abi as abi
    torch = ctx.torch
    X = gen(torch, (L, C), "normal", 3, torch.float16, 2.0 if op == "softmax" else 1.0)
    W = (gen(torch, (C,), "normal", 4, None, 0.1) + 1.0).half()
    Y = torch.empty_like(X)
    if op == "softmax":
        step = lambda: abi.softmax_f16(X, Y)  # noqa: E731
        nbytes = 2 * L * C * 2
    elif op == "rmsnorm":
        step = lambda: abi.rmsnorm_f16(X, W, Y, 1e-5)  # noqa: E731
        nbytes = 2 * L * C * 2 + C * 2
    elif op == "reduce":
        Yr = torch.empty((L,), dtype=torch.float16, device="cuda")
        step = lambda: abi.reduce_f16(X, Yr)  # noqa: E731
        nbytes = L * C * 2 + L * 2
    else:
        step = lambda: abi.channelscale_f16(X, W, Y)  # noqa: E731
        nbytes = 2 * L * C * 2 + C * 2
    ms = ctx.time_steps(step, steps, warmup)
    return {"ms": ms, "value": nbytes / ms / 1e6}


def bench_conv_f16(ctx, steps, warmup, N=32, Cc=256, H=56, W=56, Oc=256, pad=1):
    """The BASELINE conv shape in fp16 (kind::f16 MMAs on SM pairs)."""
    import unikern_b200.abi as abi
    torch = ctx.torch
    x = gen(torch, (N, Cc, H, W), "uniform", 8).half()
    w = gen(torch, (Oc, Cc, 3, 3), "normal", 9, None, (2.0 / (9 * Cc)) ** 0.5).half()
    s = gen(torch, (Oc,), "uniform", 10, None, lo=0.5, hi=1.5).half()
    y = torch.empty((N, Oc, H, W), dtype=torch.float16, device="cuda")
    n = abi.lib().uk_cuda_conv2d_f16_workspace_size(N, H, W, Cc, 3, 3, Oc, pad, abi.UK_CONV_NCHW)
    ws = torch.empty(((n + 15) // 16) * 4, dtype=torch.float32, device="cuda")
    step = lambda: abi.conv2d_f16(x, w, y, N, H, W, Cc, 3, 3, Oc, pad, s, abi.UK_CONV_NCHW, ws)  # noqa: E731
    ms = ctx.time_steps(step, steps, warmup)
    flops = 2.0 * N * H * W * Cc * 9 * Oc
    return {"ms": ms, "value": flops / ms / 1e9}


def bench_conv_sharded(ctx, steps, warmup, N=32, Cc=256, H=56, W=56, Oc=256, pad=1):
    """BASELINE configs[2] over the ranks: images split by batch, tensor-core
    conv per rank, NCCL all-gather of Y (every rank ends with the full Y)."""
    from unikern_b200 import shard
    torch = ctx.torch
    plan = shard.ConvBatchShard(N, Cc, H, W, Oc, 3, 3, pad)
    x = gen(torch, (N, Cc, H, W), "uniform", 8)[plan.b0:plan.b1].contiguous()
    w = gen(torch, (Oc, Cc, 3, 3), "normal", 9, None, (2.0 / (9 * Cc)) ** 0.5)
    s = gen(torch, (Oc,), "uniform", 10, None, lo=0.5, hi=1.5)
    y = torch.empty((N, Oc, H, W), device="cuda")
    ms = ctx.time_steps(lambda: plan.run(x, w, y, s), steps, warmup)
    flops = 2.0 * N * H * W * Cc * 9 * Oc
    return {"ms": ms, "value": flops / ms / 1e9, "parallelism": plan.describe()}


def bench_decode_sharded(ctx, steps, warmup, Bt=32, H=4096, F=14336, heads=32, S=8192):
    """BASELINE configs[4] over the ranks: weight columns sharded with the
    all-gather fused into the GEMM's store; the softmax rows split over the
    ranks (independent rows, no exchange)."""
    import unikern_b200.abi as abi
    from unikern_b200 import shard
    torch = ctx.torch
    x = gen(torch, (Bt, H), "normal", 13)
    g = gen(torch, (H,), "normal", 14, None, 0.1) + 1.0
    out = torch.empty((Bt, F), dtype=torch.float16, device="cuda")
    plan = shard.DecodeColumnShard(out, Bt, F, H)
    Ws = gen(torch, (H, F), "normal", 15, torch.float16, 0.02)[:, plan.n0:plan.n1].contiguous()
    r0, r1 = shard.batch_split(Bt * heads, ctx.world, ctx.rank)
    sc = gen(torch, (r1 - r0, S), "normal", 16)
    pr = torch.empty_like(sc)

    side = torch.cuda.Stream()

    def chain():
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            abi.softmax(sc, pr)
        plan.launch(x, g, Ws)
        torch.cuda.current_stream().wait_stream(side)

    # the kernels run as one CUDA graph per step (softmax on a parallel
    # branch); the cross-rank barrier (an NCCL all-reduce) stays outside it
    graph = capture(ctx, chain)

    def step():
        graph.replay()
        plan.barrier()
    ms = ctx.time_steps(step, steps, warmup)
    nbytes = Bt * H * 4 + H * 4 + H * F * 2 + Bt * F * 2 + 2 * Bt * heads * S * 4
    del graph
    plan.close()
    return {"ms": ms, "value": nbytes / ms / 1e6, "parallelism": plan.describe(), "graph": True}


# DRAM bytes (read + write) per launch of the dominant kernel, from one ncu
# capture of `python bench.py --op <op> --steps 2 --warmup 3 --no-cpu` with
# --metrics dram__bytes_read.sum,dram__bytes_write.sum (profiles/dram_traffic_per_kernel.md)
NCU_TRAFFIC = {
    "gemm_f16_8192x8192x8192_n1": 1255296768 + 126162944,  # k_gemm_f16_tc2 (profiles/launches_gemm_f16_8192.md)
    "rowop_reduce": 536887296 + 3104256,
    "rowop_rmsnorm": 536972800 + 480955136,
    "rowop_softmax": 536904448 + 484363008,
    "rowop_channelscale": 537094912 + 489366272,
    "rowop_reduce_scalar": 536998144 + 3074048,
}


def traffic_for(kernel_key):
    return NCU_TRAFFIC.get(kernel_key)


def roofline(bound, achieved, pk, traffic=None):
    if bound == "tensor":
        peak, unit, src = pk.get("bf16_tflops", FALLBACK["bf16_tflops"]), "TFLOP/s", pk["source"] + " bf16 burst"
    elif bound == "fp32":
        peak, unit, src = FP32_SIMT_TFLOPS, "TFLOP/s", "nominal FFMA"
    elif bound == "tensor_3xtf32":
        # fp32-accurate split-tf32: 3 tf32 MMAs per product at half the bf16
        # rate -> one sixth of the measured bf16 peak, in fp32-equivalent flop/s
        peak = round(pk.get("bf16_tflops", FALLBACK["bf16_tflops"]) / 6.0, 2)
        unit, src = "TFLOP/s", pk["source"] + " bf16 burst / 6 (3 tf32 MMAs at half rate)"
    else:
        peak, unit, src = pk.get("hbm_gbs", FALLBACK["hbm_gbs"]), "GB/s", pk["source"] + " copy"
    return {"bound": "tensor" if bound.startswith("tensor") else ("hbm" if bound == "hbm" else "fp32"),
            "achieved": round(achieved, 2), "peak": peak, "unit": unit, "frac": round(achieved / peak, 4),
            "peak_source": src, "traffic": traffic, "scope": "one launch of the kernel on one GPU"}


NVLINK_GBS = 770.0  # measured peer copy per direction per GPU on this pool (900 nominal)


def fused_roofline(g, M, N, K, world, pk):
    """Roofline of the N-sharded GEMM with the all-gather fused into its store:
    the target time per launch is the slower of its flops at the measured
    bf16 peak and the bytes it must push over NVLink (its C block to every
    peer: M * N/world * 2 B * (world - 1)) at the measured 770 GB/s per
    direction; frac = target / measured kernel time."""
    peak = pk.get("bf16_tflops", FALLBACK["bf16_tflops"])
    flops = 2.0 * M * (N / world) * K
    link_bytes = M * (N / world) * 2.0 * (world - 1)
    t_tensor = flops / (peak * 1e12) * 1e3
    t_link = link_bytes / (NVLINK_GBS * 1e9) * 1e3
    target = max(t_tensor, t_link)
    return {"bound": "tensor" if t_tensor >= t_link else "nvlink", "achieved": round(g["kernel_tflops"], 2),
            "peak": peak, "unit": "TFLOP/s", "frac": round(target / g["kernel_ms"], 4),
            "peak_source": "%s bf16 burst; NVLink %.0f GB/s per direction (measured peer copy)" % (pk["source"],
                                                                                                 NVLINK_GBS),
            "target_ms": round(target, 5), "tensor_ms": round(t_tensor, 5), "nvlink_ms": round(t_link, 5),
            "nvlink_bytes_per_launch": link_bytes, "kernel_ms": round(g["kernel_ms"], 5), "traffic": None,
            "scope": "one launch of this rank's fused GEMM + all-gather kernel"}


def run_reference(args, world, rank):
    """Reference arm: the reference's CPU implementation of the headline op."""
    if rank != 0:
        return 0
    M = N = K = 8192
    vals, last = [], None
    for i in range(args.warmup + args.steps):
        r = cpu_gemm_f16(M, N, K)
        if i >= args.warmup:
            vals.append(r["value"])
            last = r
    v = statistics.mean(vals)
    ms = 2.0 * M * N * K / (v * 1e12) * 1e3
    line = {"impl": "reference", "metric": METRIC, "value": round(v, 6), "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f16", "data": "synthetic (seeded N(0,0.02) fp16)",
            "config": {"workload": "f16 GEMM 8192^3 (reference CPU cpu_ref loop, sampled rows)", "M": M, "N": N,
                       "K": K},
            "cpu_baseline": {k: last[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": round(v, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    line["cpu_baseline"]["value"] = round(v, 6)
    print(json.dumps(line), flush=True)
    return 0


def run_single(args, ctx, pk):
    """One op alone at its BASELINE size (used for per-op numbers and profiling)."""
    op = args.op
    extra = {}
    if op in ("reduce", "rmsnorm", "softmax", "channelscale", "reduce_scalar"):
        r = bench_rowop(ctx, op, args.steps, args.warmup)
        val, unit, bound = r["value"], "GB/s", "hbm"
    elif op == "conv":
        r = bench_conv(ctx, args.steps, args.warmup)
        val, unit, bound = r["value"], "TFLOP/s", "tensor_3xtf32"
    elif op in ("softmax_f16", "rmsnorm_f16", "channelscale_f16", "reduce_f16"):
        r = bench_rowop_f16(ctx, op[:-4], args.steps, args.warmup)
        val, unit, bound = r["value"], "GB/s", "hbm"
    elif op == "conv_f16":
        r = bench_conv_f16(ctx, args.steps, args.warmup)
        val, unit, bound = r["value"], "TFLOP/s", "tensor"
    elif op == "gemm_f32":
        r = bench_gemm_f32(ctx, args.steps, args.warmup)
        val, unit, bound = r["value"], "TFLOP/s", "fp32"
    elif op == "gemm_f32_tc":
        M, N, K = (int(v) for v in args.gemm_shape.split(","))
        r = bench_gemm_f32_tc(ctx, args.steps, args.warmup, M, N, K)
        val, unit, bound = r["value"], "TFLOP/s", "tensor_3xtf32"
        extra = {"config": {"workload": "fp32 GEMM %dx%dx%d, split-tf32 tensor cores, pre-passes included" % (M, N, K)}}
    elif op in ("gemm_streamed", "gemm_streamed_f16"):
        M, N, K = (int(v) for v in args.gemm_shape.split(",")) if args.gemm_shape != "8192,8192,8192" else \
            (32768, 32768, 32768)
        r = bench_gemm_streamed(ctx, args.steps, args.warmup, M, N, K, f16=op.endswith("f16"))
        val, unit, bound = r["value"], "TFLOP/s", "tensor" if op.endswith("f16") else "tensor_3xtf32"
        es = 2 if op.endswith("f16") else 4
        extra = {"e2e": {"value": round(val, 3), "unit": unit, "h2d_bytes_per_step": (M * K + K * N) * es,
                         "d2h_bytes_per_step": M * N * es},
                 "config": {"workload": "GEMM %dx%dx%d %s streamed from pinned host memory, B resident, %d row "
                                        "blocks in a two-slot ring" % (M, N, K, "f16" if es == 2 else "fp32",
                                                                       r["blocks"])},
                 "host_link_GBps": round(r["link_GBps"], 2), "seconds_per_step": round(r["ms"] / 1e3, 4)}
    else:
        r = bench_decode(ctx, args.steps, args.warmup)
        val, unit, bound = r["value"], "GB/s", "hbm"
    if ctx.rank == 0:
        line = {"metric": METRIC, "op": op, "value": round(val, 3), "unit": unit, "n_gpus": ctx.world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(r["ms"], 5),
                "higher_is_better": True, "roofline": roofline(bound, val, pk)}
        line.update(extra)
        print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--op", default="all",
                    choices=["all", "gemm_f16", "reduce", "rmsnorm", "softmax", "channelscale", "reduce_scalar",
                             "conv", "gemm_f32", "decode", "softmax_f16", "rmsnorm_f16", "channelscale_f16",
                             "conv_f16", "gemm_streamed", "gemm_streamed_f16", "gemm_f32_tc", "reduce_f16"],
                    help="all = headline f16 GEMM + every other op; otherwise one op alone (profiling)")
    ap.add_argument("--gemm-shape", default="8192,8192,8192", help="M,N,K of the f16 GEMM")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline legs")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, world, rank)

    import torch
    torch.cuda.set_device(local_rank)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                             device_id=torch.device("cuda", local_rank))
    import unikern_b200.abi as abi
    abi.lib()
    ctx = Ctx(world, rank, local_rank)
    pk = peaks()

    if args.op not in ("all", "gemm_f16"):
        return run_single(args, ctx, pk)
    M, N, K = (int(v) for v in args.gemm_shape.split(","))
    sampler = ClockSampler(local_rank)
    sampler.start()
    g = bench_gemm_f16(ctx, args.steps, args.warmup, M, N, K)
    clocks = sampler.stop()

    ops = {}
    if args.op == "all" and world == 1:
        s = max(5, min(args.steps, 20))
        for op in ("reduce", "rmsnorm", "softmax", "channelscale", "reduce_scalar"):
            r = bench_rowop(Ctx(1, 0, local_rank), op, s, 3)
            ops[op] = {"GB/s": round(r["value"], 1), "ms": round(r["ms"], 4),
                       "roofline": roofline("hbm", r["value"], pk, traffic_for("rowop_" + op))}
        r = bench_conv(Ctx(1, 0, local_rank), max(3, s // 2), 3)
        ops["conv_n32_256_56_3x3_pad1_scaled"] = {
            "TFLOP/s": round(r["value"], 2), "ms": round(r["ms"], 4),
            "path": "split-tf32 (3xTF32) implicit GEMM on tcgen05; the step includes the NCHW->NHWC hi/lo pre-pass",
            "roofline": roofline("tensor_3xtf32", r["value"], pk)}
        r = bench_gemm_f32(Ctx(1, 0, local_rank), s, 3)
        ops["gemm_f32_512"] = {"TFLOP/s": round(r["value"], 3), "ms": round(r["ms"], 5),
                               "roofline": roofline("fp32", r["value"], pk)}
        r = bench_decode(Ctx(1, 0, local_rank), s, 3)
        ops["decode_chain_b32"] = {"GB/s": round(r["value"], 1), "ms": round(r["ms"], 4),
                                   "roofline": roofline("hbm", r["value"], pk)}
        # fp16 variants (beyond the reference's dtype interval)
        for op in ("softmax", "rmsnorm", "channelscale", "reduce"):
            r = bench_rowop_f16(Ctx(1, 0, local_rank), op, s, 3)
            ops[op + "_f16"] = {"GB/s": round(r["value"], 1), "ms": round(r["ms"], 4),
                                "roofline": roofline("hbm", r["value"], pk)}
        r = bench_conv_f16(Ctx(1, 0, local_rank), max(3, s // 2), 3)
        ops["conv_f16_n32_256_56_3x3_pad1_scaled"] = {"TFLOP/s": round(r["value"], 2), "ms": round(r["ms"], 4),
                                                     "roofline": roofline("tensor", r["value"], pk)}
        # last: the only op that holds ~3 GB and runs seconds-long tensor-core
        # work; it runs after the memory-bound ops so it cannot perturb them
        r = bench_gemm_f32_tc(Ctx(1, 0, local_rank), max(3, s // 2), 3)
        ops["gemm_f32_8192_tensor_cores"] = {
            "TFLOP/s": round(r["value"], 2), "ms": round(r["ms"], 4),
            "path": "split-tf32 on the convolution's SM-pair kernel, fp32 promotion every 1024 k; pre-passes included",
            "roofline": roofline("tensor_3xtf32", r["value"], pk)}
        if not args.no_cpu:
            # the reference's CPU path for every op, timed on this host in this run
            for op in ("reduce", "rmsnorm", "softmax", "channelscale"):
                ops[op]["cpu_baseline"] = strip(cpu_rowop(op, 8192, 16384))
            ops["reduce_scalar"]["cpu_baseline"] = strip(cpu_reduce_scalar())
            ops["conv_n32_256_56_3x3_pad1_scaled"]["cpu_baseline"] = strip(cpu_conv(32, 256, 56, 56, 256, 1))
            ops["gemm_f32_512"]["cpu_baseline"] = strip(cpu_gemm_f32())
            ops["decode_chain_b32"]["cpu_baseline"] = strip(cpu_decode())

    if args.op == "all" and world > 1:
        r = bench_conv_sharded(ctx, max(3, min(args.steps, 10)), 3)
        ops["conv_n32_batch_sharded"] = {"TFLOP/s": round(r["value"], 2), "ms": round(r["ms"], 4),
                                         "parallelism": r["parallelism"], "scaling": "strong"}
        r = bench_decode_sharded(ctx, max(5, min(args.steps, 20)), 3)
        ops["decode_chain_b32_column_sharded"] = {"GB/s": round(r["value"], 1), "ms": round(r["ms"], 4),
                                                  "parallelism": r["parallelism"], "scaling": "strong"}

    tflops = g["value"]
    line = {"metric": METRIC, "value": round(tflops, 3), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(g["ms"], 5), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic (seeded N(0,0.02) fp16 on device)",
            "config": {"workload": "f16 GEMM C=A*B, f32 accumulation, f16 out, M=%d N=%d K=%d row-major "
                                   "(BASELINE configs[3])" % (M, N, K), "M": M, "N": N, "K": K,
                       "parallelism": g["parallelism"], "l2": "inputs (256 MiB) larger than L2"},
            "roofline": roofline("tensor", g["kernel_tflops"], pk,
                                 traffic_for("gemm_f16_%dx%dx%d_n%d" % (M, N, K, world))) if world == 1 else
            fused_roofline(g, M, N, K, world, pk),
            "e2e": {k: (round(v, 3) if isinstance(v, float) else v) for k, v in g["e2e"].items()},
            "gpu_launches": g["launches"], "clocks": clocks}
    line["e2e"]["value"] = round(g["e2e"]["value"], 3)
    if "allgather_max_abs_diff" in g:
        line["config"]["allgather_check_max_abs_diff"] = g["allgather_max_abs_diff"]
    if world == 1 and not args.no_cpu:
        cb = cpu_gemm_f16(M, N, K, rows=10 * cpu_threads())  # ~10 s of host work
        line["cpu_baseline"] = {k: (round(v, 6) if isinstance(v, float) else v) for k, v in cb.items()
                                if k != "seconds"}
    if ops:
        line["ops"] = ops
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
