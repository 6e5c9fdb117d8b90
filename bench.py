#!/usr/bin/env python
"""bench.py -- throughput of the B200 KML operator set (JSON lines, headline last).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--op OP]

Headline workload (``value``, the LAST line): f16 GEMM, C(f16) = A(f16) * B(f16)
with f32 accumulation, M = N = K = 8192 row-major; at N
GPUs the columns of B and C are split over the ranks (strong scaling, total
work fixed).  A step is one GEMM over inputs already resident in HBM; ``e2e``
is the same metric through the C ABI with pinned host buffers copied in and
the result copied out inside the timed region.

Before the headline, one compact JSON line per other BASELINE op (rank 0,
one GPU): the f32 GEMM 512^3, the row reduce, the KML scalar reduce, RMSNorm
and softmax over [8192 x 16384], the conv N=32 256->256 56x56 3x3 pad 1 with
the fused channel scale (split-tf32 tensor cores, with the FFMA kernel
beside it) and the decode chain.  Each carries ``roofline``, ``e2e`` (the op
through the C ABI with its inputs uploaded from and its outputs downloaded to
pinned host memory inside the timed region, the reference's measured_ms,
src/codegen_hip.cpp:692-744) and ``cpu_baseline`` (the reference's CPU code on
this host's cores).  The fp16 widenings and channelscale print first.  Just
before the headline, one short `baseline_rows` line repeats every BASELINE
row's value, unit, roofline fraction, e2e and CPU baseline, so that all of
them sit with the headline in the last ~1.5 KB of the output.

Timing: W untimed steps, then exactly K steps between CUDA events on the
launching stream, barrier + synchronize on both sides, max over ranks.
Inputs are larger than L2 (126 MB) for every HBM-bound op and the GEMM; the
f32 GEMM 512^3, whose inputs fit in L2, writes a 256 MiB buffer before each
step (outside the timed interval) and times each step between its own events.
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
import warnings
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
warnings.filterwarnings("ignore")  # stdout/stderr carry the JSON lines only

METRIC = json.loads((ROOT / "BASELINE.json").read_text())["metric"] if (ROOT / "BASELINE.json").exists() else \
    "f16 GEMM TFLOP/s; reduce/norm/softmax HBM GB/s; % roofline at 1/2/4/8 B200"
FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
FP32_SIMT_TFLOPS = 2 * 148 * 128 * 1.965e9 / 1e12  # nominal FFMA peak (no measured figure exists)
SUSTAINED_LAUNCHES = 2000  # the headline GEMM back to back for ~1.7 s (burst vs power-capped clocks)


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        d["source"] = "measured"
        return d
    d = dict(FALLBACK)
    d["source"] = "fallback"
    return d


def emit(d):
    print(json.dumps(d, separators=(",", ":")), flush=True)


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
        return self

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

    def time_steps_flushed(self, step, steps, warmup):
        """ms per step for an op whose inputs fit in L2: before every step a
        256 MiB buffer (larger than the 126 MB L2) is written, outside the
        timed interval, and each step is timed between its own pair of CUDA
        events on the launching stream (the flush ahead of it also keeps the
        GPU from waiting on the host's launch of the step).  Mean over exactly
        `steps` steps, max over ranks."""
        torch = self.torch
        if getattr(self, "_flush", None) is None:
            self._flush = torch.empty(64 << 20, dtype=torch.float32, device="cuda")
        for _ in range(warmup):
            self._flush.zero_()
            step()
        torch.cuda.synchronize()
        self.barrier()
        torch.cuda.synchronize()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for e0, e1 in evs:
            self._flush.zero_()
            e0.record(self.stream)
            step()
            e1.record(self.stream)
        torch.cuda.synchronize()
        self.barrier()
        torch.cuda.synchronize()
        return self.max_over_ranks(sum(e0.elapsed_time(e1) for e0, e1 in evs) / steps)

    def time_steps(self, step, steps, warmup):
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


def pinned(t):
    """A page-locked host copy of device tensor t."""
    return t.cpu().pin_memory()


def time_e2e(ctx, launch, ins, outs, steps, warmup=3):
    """The op end to end, as the reference's measured_ms: every step uploads
    each (device, pinned host) pair of `ins`, launches, and downloads each
    pair of `outs`, all on the launching stream between CUDA events.
    Returns (ms per step, H2D bytes per step, D2H bytes per step)."""
    def step():
        for d, h in ins:
            d.copy_(h, non_blocking=True)
        launch()
        for d, h in outs:
            h.copy_(d, non_blocking=True)
    ms = ctx.time_steps(step, steps, warmup)
    nb = lambda pairs: sum(h.numel() * h.element_size() for _, h in pairs)  # noqa: E731
    return ms, nb(ins), nb(outs)


def e2e_record(work, unit, ms, h2d, d2h):
    """work per step (bytes for GB/s, flops for TFLOP/s) over the e2e time."""
    v = work / ms / (1e6 if unit == "GB/s" else 1e9)
    return {"value": round(v, 3), "h2d": h2d, "d2h": d2h}


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


def gemm_f16_cpu_rows():
    """Rows of the 8192^3 product the CPU baseline computes; the headline's
    cpu_baseline and the reference arm use the same count."""
    return 4 * cpu_threads()


_CPU_B = {}


def cpu_gemm_f16(M, N, K, rows=None):
    """Rows of C = A * B (8192^3 f16 config) with the reference's cpu_ref loop
    (src/codegen_hip.cpp:1124-1132 on half-quantised inputs); rows dealt
    round-robin over the host threads."""
    import numpy as np
    from oracle import oracle as O
    nt = cpu_threads()
    e = O.emit()
    kind = "reference" if e is not None else "port"
    # B (and the reference library's copy of it) is made once per shape and
    # reused by every later call: a step times only its sampled rows
    key = (K, N)
    if _CPU_B.get("key") != key:
        rng = np.random.default_rng(5)
        _CPU_B.update(key=key, Bh=O.f32_to_f16(rng.normal(0, 0.02, (K, N)).astype(np.float32)), loaded=False)
    Bh = _CPU_B["Bh"]
    nrows = rows or gemm_f16_cpu_rows()
    rng = np.random.default_rng(6 + nrows)
    Ah = O.f32_to_f16(rng.normal(0, 0.02, (nrows, K)).astype(np.float32))
    if e is not None:
        if not _CPU_B["loaded"]:
            e.emit_gemm_set_B(O.f16_to_f32(Bh), K, N)
            _CPU_B["loaded"] = True
        Af = O.f16_to_f32(Ah)
        out = np.zeros((nrows, N), np.float32)

        def work(t):  # thread t takes rows t, t + nt, ...
            for i in range(t, nrows, nt):
                e.emit_gemm_f16_rows(Af[i:i + 1].copy(), out[i:i + 1], 1)
        dt = run_threads(work, min(nt, nrows))
    else:
        t0 = time.perf_counter()
        O.gemm_f16(Ah, Bh, threads=nt)
        dt = time.perf_counter() - t0
    flops = 2.0 * nrows * N * K
    return {"value": flops / dt / 1e12, "unit": "TFLOP/s", "cores": min(nt, nrows), "kind": kind,
            "sample": "%d rows of C, %.2f s, extrapolated by rate" % (nrows, dt), "seconds": dt}


def cpu_rowop(op, L, C):
    """The whole [L x C] workload with the reference's CPU code, one block of
    rows per host thread."""
    import numpy as np
    from oracle import oracle as O
    nt = cpu_threads()
    rows = L
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
            "sample": "all %d rows (C=%d), %.2f s%s" % (rows, C, dt, "; eps 1e-6" if op == "rmsnorm" else ""),
            "short": "all rows" + (", eps 1e-6" if op == "rmsnorm" else ""), "seconds": dt}


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
            "sample": "%d of %d images, %.2f s" % (nt, N, dt), "short": "%d images, by rate" % nt, "seconds": dt}


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
            "sample": "whole %d^3 GEMM, %.3f s" % (M, dt), "short": "whole", "seconds": dt}


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
            "sample": "whole vector L=%d, %.3f s" % (L, dt), "short": "whole, 1 thread", "seconds": dt}


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
            "sample": "whole chain B=%d, %.3f s" % (Bt, dt), "short": "whole", "seconds": dt}


def cpu_short(d):
    """The cpu_baseline object of a per-op line."""
    if d is None:
        return None
    return {"value": round(d["value"], 6), "cores": d["cores"], "kind": d["kind"], "sample": d["short"]}


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


def check_gemm_f16(A, B, Cm, rows, points=0, seed=0):
    """Sampled check of a computed C against float64 dot products of the half
    inputs (numpy on the host; a checker beside the timing, never timed):
    `rows` full rows of C (every rank's column block) and `points` random
    elements.  Returns the worst |C - ref| / max(|ref|, RMS(ref))."""
    import numpy as np
    M, N = Cm.shape
    rng = np.random.default_rng(seed)
    idx = np.unique(np.concatenate([[0, M - 1], rng.choice(M, max(0, rows - 2), replace=False)]))
    Bf = B.double().cpu().numpy()
    ref = A[idx].double().cpu().numpy() @ Bf
    got = Cm[idx].double().cpu().numpy()
    tau = float(np.sqrt(np.mean(ref * ref)))
    err = float(np.max(np.abs(got - ref) / np.maximum(np.abs(ref), tau)))
    if points:
        import torch
        i = rng.integers(0, M, points)
        j = rng.integers(0, N, points)
        refp = np.einsum("pk,kp->p", A[i].double().cpu().numpy(), Bf[:, j])
        gotp = Cm[torch.as_tensor(i, device=Cm.device), torch.as_tensor(j, device=Cm.device)].double().cpu().numpy()
        err = max(err, float(np.max(np.abs(gotp - refp) / np.maximum(np.abs(refp), tau))))
    return err, len(idx)


def bench_gemm_f16(ctx, steps, warmup, M=8192, N=8192, K=8192, profile_only=False):
    import unikern_b200.abi as abi
    torch = ctx.torch
    world, rank = ctx.world, ctx.rank
    A = gen(torch, (M, K), "normal", 1, torch.float16, 0.02)
    B = gen(torch, (K, N), "normal", 2, torch.float16, 0.02)
    Cm = torch.empty((M, N), dtype=torch.float16, device="cuda")
    plan = None
    if world == 1:
        def launch():
            abi.gemm_f16(A, B, Cm)
        step = launch
        launches_per_step = 1
        parallelism = "single GPU"
        Bs = B
    else:
        from unikern_b200 import shard
        plan = shard.GemmAllGather(Cm, M, N, K)
        Bs = plan.b_shard(B)

        def launch():
            plan.launch(A, Bs)

        def step():
            launch()
            plan.barrier()
        launches_per_step = plan.launches_per_step
        parallelism = plan.describe()
    sampler = ClockSampler(ctx.local_rank).start()
    ms = ctx.time_steps(step, steps, warmup)
    clocks = sampler.stop()
    # the dominant kernel's own launch time: events on the launching stream
    # around each GEMM alone (at N > 1 the barrier falls outside), max over ranks
    kev = []
    for _ in range(steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(ctx.stream)
        launch()
        e1.record(ctx.stream)
        kev.append((e0, e1))
        if plan is not None:
            plan.barrier()
    torch.cuda.synchronize()
    kernel_ms = ctx.max_over_ranks(sum(a.elapsed_time(b) for a, b in kev) / len(kev))
    flops = 2.0 * M * N * K
    flops_per_launch = flops if world == 1 else 2.0 * M * (plan.n1 - plan.n0) * K
    res = {"ms": ms, "value": flops / ms / 1e9, "flops_per_step": flops, "launches": launches_per_step * steps,
           "parallelism": parallelism, "kernel_ms": kernel_ms, "kernel_tflops": flops_per_launch / kernel_ms / 1e9,
           "clocks": clocks}

    if profile_only:  # --no-e2e: the timed steps alone (ncu captures of this kernel)
        if plan is not None:
            plan.close()
        return res
    # sustained: the same step back to back for ~1.7 s with clocks sampled,
    # so the power-capped rate is measured beside the burst figure above
    sampler = ClockSampler(ctx.local_rank).start()
    sms = ctx.time_steps(step, SUSTAINED_LAUNCHES, 0)
    sclk = sampler.stop()
    res["sustained"] = {"launches": SUSTAINED_LAUNCHES, "value": round(flops / sms / 1e9, 2),
                        "sm_mhz": sclk["sm_mhz"] if sclk else None,
                        "reasons": sclk["reasons"] if sclk else None}

    # e2e through the C ABI with pinned host buffers: on one GPU the pipelined
    # host-to-host entry point (uploads of A row blocks, their GEMMs and the
    # downloads of C blocks overlapped); on N GPUs the sharded host path
    if world == 1:
        Ah, Bh = pinned(A), pinned(B)
        Ch = torch.empty((M, N), dtype=torch.float16).pin_memory()
        Bd = torch.empty_like(B)
        e2e_step = lambda: abi.gemm_f16_host(Ah, Bh, Ch, A, Bd, Cm)  # noqa: E731
        h2d, d2h = Ah.numel() * 2 + Bh.numel() * 2, Ch.numel() * 2
    else:
        host = shard.HostGemmF16(plan, A, B)
        e2e_step = host.step
        h2d, d2h = host.h2d_bytes, host.d2h_bytes
    e2e_ms = ctx.time_steps(e2e_step, max(3, min(steps, 10)), 3)
    res["e2e"] = {"value": round(flops / e2e_ms / 1e9, 3), "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                  "d2h_bytes_per_step": d2h}
    if world > 1:
        # the host C the sharded e2e path assembled: every rank's block
        res["e2e"]["check"] = host.check_host(step_fn=e2e_step)
        host.close()

    # correctness of the timed product (a checker, after the timing): at N=1
    # 64 full rows + 4096 elements, at N>1 16 full rows of this rank's gathered
    # C (every rank's column block), each against float64 dot products; max over ranks
    step()
    torch.cuda.synchronize()
    err, nrows = check_gemm_f16(A, B, Cm, 64 if world == 1 else 16, 4096 if world == 1 else 0, seed=rank)
    err = ctx.max_over_ranks(err)
    res["check"] = {"rows": nrows, "points": 4096 if world == 1 else 0, "err_vs_f64": float("%.3g" % err),
                    "pass": err <= 2e-2}
    if plan is not None:
        plan.close()
    return res


def rowop_tensors(torch, op, L=8192, C=16384):
    X = gen(torch, (L, C), "normal", 3, None, 2.0 if op == "softmax" else 1.0)
    W = gen(torch, (C,), "normal", 4, None, 0.1) + 1.0
    return X, W


def measure_rowop(ctx, op, steps, warmup, pk, L=8192, C=16384, e2e=True):
    """Row reduce / RMSNorm / softmax / channelscale / KML scalar reduce at
    the BASELINE row shape: device-resident rate, then e2e."""
    import unikern_b200.abi as abi
    torch = ctx.torch
    X, W = rowop_tensors(torch, op, L, C)
    Y = torch.empty((L, C), device="cuda")
    R = torch.empty((L,), device="cuda")
    ins, outs = [(X, pinned(X))], []
    if op == "rmsnorm":
        launch = lambda: abi.rmsnorm(X, W, Y, 1e-5)  # noqa: E731
        nbytes = 2 * L * C * 4 + C * 4
        ins.append((W, pinned(W)))
        outs.append((Y, torch.empty_like(Y, device="cpu").pin_memory()))
    elif op == "softmax":
        launch = lambda: abi.softmax(X, Y)  # noqa: E731
        nbytes = 2 * L * C * 4
        outs.append((Y, torch.empty_like(Y, device="cpu").pin_memory()))
    elif op == "channelscale":
        launch = lambda: abi.channelscale(X, W, Y)  # noqa: E731
        nbytes = 2 * L * C * 4 + C * 4
        ins.append((W, pinned(W)))
        outs.append((Y, torch.empty_like(Y, device="cpu").pin_memory()))
    elif op == "reduce":
        launch = lambda: abi.reduce(X, R)  # noqa: E731
        nbytes = L * C * 4 + L * 4
        outs.append((R, torch.empty_like(R, device="cpu").pin_memory()))
    else:  # reduce_scalar: the KML reduce, one vector of L*C floats to a scalar
        Xs = X.view(1, L * C)
        ws = torch.empty(max(1, abi.reduce_workspace_size(1, L * C) // 4), device="cuda")
        launch = lambda: abi.reduce(Xs, R[:1], ws)  # noqa: E731
        nbytes = L * C * 4 + 4
        outs.append((R[:1], torch.empty(1).pin_memory()))
    ms = ctx.time_steps(launch, steps, warmup)
    val = nbytes / ms / 1e6
    rec = {"value": val, "unit": "GB/s", "ms": ms, "bytes_per_step": nbytes,
           "roofline": roofline("hbm", val, pk, traffic_for("rowop_" + op))}
    if e2e:
        if op == "reduce_scalar":  # one row: upload, reduce, download in turn
            ems, h2d, d2h = time_e2e(ctx, launch, ins, outs, max(3, min(steps, 10)))
        else:  # uk_cuda_rowop_host: row blocks pipelined, both link directions at once
            Xh = ins[0][1]
            Wh = ins[1][1] if len(ins) > 1 else None
            Yd, Yh = outs[0]
            ems = ctx.time_steps(lambda: abi.rowop_host(op, Xh, Wh, Yh, X, W if Wh is not None else None, Yd,
                                                        1e-5), max(3, min(steps, 10)), 3)
            h2d = sum(h.numel() * h.element_size() for _, h in ins)
            d2h = Yh.numel() * Yh.element_size()
        rec["e2e"] = e2e_record(nbytes, "GB/s", ems, h2d, d2h)
    return rec


def conv_tensors(torch, N=32, Cc=256, H=56, W=56, Oc=256):
    x = gen(torch, (N, Cc, H, W), "uniform", 8)
    w = gen(torch, (Oc, Cc, 3, 3), "normal", 9, None, (2.0 / (9 * Cc)) ** 0.5)
    s = gen(torch, (Oc,), "uniform", 10, None, lo=0.5, hi=1.5)
    return x, w, s


def measure_conv(ctx, steps, warmup, pk, N=32, Cc=256, H=56, W=56, Oc=256, pad=1, ffma=True, e2e=True):
    """the split-tf32 tensor-core conv (step includes its
    NCHW->NHWC hi/lo pre-pass) and, beside it, the FFMA kernel the north star
    names for the fp32 path."""
    import unikern_b200.abi as abi
    torch = ctx.torch
    x, w, s = conv_tensors(torch, N, Cc, H, W, Oc)
    y = torch.empty((N, Oc, H, W), device="cuda")
    ws = abi.conv2d_workspace(N, H, W, Cc, 3, 3, Oc, pad, abi.UK_CONV_NCHW)
    launch = lambda: abi.conv2d_tc(x, w, y, N, H, W, Cc, 3, 3, Oc, pad, s, abi.UK_CONV_NCHW, ws)  # noqa: E731
    ms = ctx.time_steps(launch, steps, warmup)
    flops = 2.0 * N * H * W * Cc * 9 * Oc
    val = flops / ms / 1e9
    rec = {"value": val, "unit": "TFLOP/s", "ms": ms, "path": "3xTF32 tcgen05 SM pairs",
           "roofline": roofline("tensor_3xtf32", val, pk)}
    if e2e:
        # uk_cuda_conv2d_f32_host: the weights, then blocks of images up, each
        # block's conv, its Y down while later blocks upload
        xh, wh, sh = pinned(x), pinned(w), pinned(s)
        yh = torch.empty_like(y, device="cpu").pin_memory()
        hws_n = abi.lib().uk_cuda_conv2d_f32_host_workspace_size(N, H, W, Cc, 3, 3, Oc, pad, 0)
        hws = torch.empty(((hws_n + 15) // 16) * 4, device="cuda")
        ems = ctx.time_steps(lambda: abi.conv2d_host(xh, wh, sh, yh, x, w, s, y, N, H, W, Cc, 3, 3, Oc, pad, 0, hws),
                             max(3, min(steps, 10)), 3)
        h2d = sum(t.numel() * t.element_size() for t in (xh, wh, sh))
        rec["e2e"] = e2e_record(flops, "TFLOP/s", ems, h2d, yh.numel() * yh.element_size())
    if ffma:
        fl = lambda: abi.conv2d(x, w, y, N, H, W, Cc, 3, 3, Oc, pad, s, abi.UK_CONV_NCHW)  # noqa: E731
        fms = ctx.time_steps(fl, max(3, min(steps, 5)), 3)
        fval = flops / fms / 1e9
        rec["ffma"] = {"value": round(fval, 2), "frac": round(fval / FP32_SIMT_TFLOPS, 4)}
    return rec


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


def measure_gemm_f32(ctx, steps, warmup, pk, M=512, N=512, K=512, e2e=True):
    """the FFMA GEMM at 512^3 (a few microseconds of
    device time).  Its 3 MB of inputs fit in L2, so each device-resident step
    follows a write of a buffer larger than L2 and is timed on its own
    (time_steps_flushed); the step replays a CUDA graph of the one launch.
    e2e calls the C ABI directly, host copies inside the timed region."""
    import unikern_b200.abi as abi
    torch = ctx.torch
    A = gen(torch, (M, K), "uniform", 11, lo=-1, hi=1)
    B = gen(torch, (K, N), "uniform", 12, lo=-1, hi=1)
    Cm = torch.empty((M, N), device="cuda")
    launch = lambda: abi.gemm_f32(A, B, Cm)  # noqa: E731
    graph = capture(ctx, launch)
    ms = ctx.time_steps_flushed(graph.replay, steps, warmup)
    flops = 2.0 * M * N * K
    val = flops / ms / 1e9
    rec = {"value": val, "unit": "TFLOP/s", "ms": ms, "graph": True, "l2": "flushed before each step",
           "roofline": roofline("fp32", val, pk)}
    if e2e:
        ins = [(A, pinned(A)), (B, pinned(B))]
        outs = [(Cm, torch.empty_like(Cm, device="cpu").pin_memory())]
        ems, h2d, d2h = time_e2e(ctx, launch, ins, outs, max(10, steps))
        rec["e2e"] = e2e_record(flops, "TFLOP/s", ems, h2d, d2h)
    return rec


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


def measure_decode(ctx, steps, warmup, pk, Bt=32, H=4096, F=14336, heads=32, S=8192, e2e=True):
    """Decode-layer chain: RMSNorm [B x 4096] fused into
    the f16 skinny GEMM [B x 4096] x [4096 x 14336], then softmax over
    [B*32 x 8192] scores.  HBM-bound: the 112 MiB of weights dominate.
    e2e: the layer weight and gamma stay resident (model state); each step
    uploads the token rows and the scores and downloads the GEMM output and
    the probabilities, the scores' blocks pipelined through the softmax."""
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
    val = nbytes / ms / 1e6
    rec = {"value": val, "unit": "GB/s", "ms": ms, "graph": True, "roofline": roofline("hbm", val, pk)}
    if e2e:
        # through the C ABI: the scores' blocks go up, through the softmax and
        # back down pipelined (uk_cuda_rowop_host), and the token rows up,
        # through the norm + GEMM and the GEMM's output back down
        xh, sch = pinned(x), pinned(sc)
        outh = torch.empty_like(out, device="cpu").pin_memory()
        prh = torch.empty_like(pr, device="cpu").pin_memory()

        def e2e_step():
            abi.rowop_host("softmax", sch, None, prh, sc, None, pr, 1e-5, 8)
            x.copy_(xh, non_blocking=True)
            abi.decode_rmsnorm_gemm(x, g, Wt, out, 1e-5, ws)
            outh.copy_(out, non_blocking=True)
        ems = ctx.time_steps(e2e_step, max(5, min(steps, 20)), 3)
        h2d = sum(t.numel() * t.element_size() for t in (xh, sch))
        d2h = sum(t.numel() * t.element_size() for t in (outh, prh))
        rec["e2e"] = e2e_record(nbytes, "GB/s", ems, h2d, d2h)
    del graph
    return rec


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
    plan.close()
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
        peak, unit, src = round(FP32_SIMT_TFLOPS, 1), "TFLOP/s", "nominal FFMA"
    elif bound == "tensor_3xtf32":
        # fp32-accurate split-tf32: 3 tf32 MMAs per product at half the bf16
        # rate -> one sixth of the measured bf16 peak, in fp32-equivalent flop/s
        peak = round(pk.get("bf16_tflops", FALLBACK["bf16_tflops"]) / 6.0, 2)
        unit, src = "TFLOP/s", pk["source"] + " bf16 burst / 6"
    else:
        peak, unit, src = pk.get("hbm_gbs", FALLBACK["hbm_gbs"]), "GB/s", pk["source"] + " copy"
    return {"bound": "tensor" if bound.startswith("tensor") else ("hbm" if bound == "hbm" else "fp32"),
            "achieved": round(achieved, 2), "peak": peak, "unit": unit, "frac": round(achieved / peak, 4),
            "peak_source": src, "traffic": traffic}


def op_line(name, rec, cpu=None, **extra):
    """One compact JSON line per op: value, roofline (peak_source kept
    short), e2e and cpu_baseline."""
    roof = dict(rec["roofline"])
    for k in ("achieved", "unit", "peak_source"):  # = value, = unit, in the peaks line
        roof.pop(k, None)
    if roof.get("traffic") is None:
        roof.pop("traffic", None)
    d = {"op": name, "value": round(rec["value"], 3), "unit": rec["unit"], "ms": round(rec["ms"], 5),
         "roofline": roof}
    if "e2e" in rec:
        d["e2e"] = rec["e2e"]
    if cpu is not None:
        d["cpu_baseline"] = cpu_short(cpu)
    for k in ("ffma", "l2"):
        if k in rec:
            d[k] = rec[k]
    d.update(extra)
    return d


def summarize(rows, line):
    """Record an op line's headline figures in `rows` (for the compact
    baseline_rows line) and return the line unchanged."""
    rows[line["op"]] = [line["value"], line["unit"], line["roofline"].get("frac"),
                        (line.get("e2e") or {}).get("value"), (line.get("cpu_baseline") or {}).get("value")]
    return line


NVLINK_GBS = 770.0  # measured peer copy per direction per GPU on this pool (900 nominal)


def fused_roofline(g, M, N, K, world, pk):
    """Roofline of the N-sharded GEMM with the all-gather fused into its store:
    the target time per launch is the slower of its flops at the measured
    bf16 peak and the bytes this GPU must receive over NVLink (every peer's C
    block: M * N/world * 2 B * (world - 1)) at the measured 770 GB/s per
    direction; frac = target / measured kernel time."""
    peak = pk.get("bf16_tflops", FALLBACK["bf16_tflops"])
    flops = 2.0 * M * (N / world) * K
    link_bytes = M * (N / world) * 2.0 * (world - 1)
    t_tensor = flops / (peak * 1e12) * 1e3
    t_link = link_bytes / (NVLINK_GBS * 1e9) * 1e3
    target = max(t_tensor, t_link)
    return {"bound": "tensor" if t_tensor >= t_link else "nvlink", "achieved": round(g["kernel_tflops"], 2),
            "peak": peak, "unit": "TFLOP/s", "frac": round(target / g["kernel_ms"], 4),
            "peak_source": "%s bf16 burst; NVLink %.0f GB/s" % (pk["source"], NVLINK_GBS),
            "target_ms": round(target, 5), "tensor_ms": round(t_tensor, 5), "nvlink_ms": round(t_link, 5),
            "kernel_ms": round(g["kernel_ms"], 5), "traffic": None}


def run_reference(args, world, rank):
    """Reference arm: the reference's CPU implementation of the headline op."""
    if rank != 0:
        return 0
    M = N = K = 8192
    vals, last = [], None
    # each step samples rows of C; the sample shrinks with the step count so
    # that the whole run stays near two minutes (~0.056 s a row here), never
    # below one row per host thread and never above the headline's own count
    per_step = 120.0 / max(1, args.warmup + args.steps)
    rows = max(cpu_threads(), min(gemm_f16_cpu_rows(), int(per_step / 0.056)))
    for i in range(args.warmup + args.steps):
        r = cpu_gemm_f16(M, N, K, rows=rows)
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
    emit(line)
    return 0


SINGLE_OPS = ["gemm_f16", "reduce", "rmsnorm", "softmax", "channelscale", "reduce_scalar", "conv", "gemm_f32",
              "decode", "softmax_f16", "rmsnorm_f16", "channelscale_f16", "conv_f16", "gemm_streamed",
              "gemm_streamed_f16", "gemm_f32_tc", "reduce_f16"]


def run_single(args, ctx, pk):
    """One op alone at its BASELINE size (per-op numbers and profiling)."""
    op = args.op
    extra = {}
    if op in ("reduce", "rmsnorm", "softmax", "channelscale", "reduce_scalar"):
        r = measure_rowop(ctx, op, args.steps, args.warmup, pk, e2e=not args.no_e2e)
    elif op == "conv":
        r = measure_conv(ctx, args.steps, args.warmup, pk, ffma=not args.no_e2e, e2e=not args.no_e2e)
    elif op == "gemm_f32":
        r = measure_gemm_f32(ctx, args.steps, args.warmup, pk, e2e=not args.no_e2e)
    elif op == "decode":
        r = measure_decode(ctx, args.steps, args.warmup, pk, e2e=not args.no_e2e)
    elif op in ("softmax_f16", "rmsnorm_f16", "channelscale_f16", "reduce_f16"):
        r = bench_rowop_f16(ctx, op[:-4], args.steps, args.warmup)
        r.update(unit="GB/s", roofline=roofline("hbm", r["value"], pk))
    elif op == "conv_f16":
        r = bench_conv_f16(ctx, args.steps, args.warmup)
        r.update(unit="TFLOP/s", roofline=roofline("tensor", r["value"], pk))
    elif op == "gemm_f32_tc":
        M, N, K = (int(v) for v in args.gemm_shape.split(","))
        r = bench_gemm_f32_tc(ctx, args.steps, args.warmup, M, N, K)
        r.update(unit="TFLOP/s", roofline=roofline("tensor_3xtf32", r["value"], pk))
        extra = {"config": {"workload": "fp32 GEMM %dx%dx%d, split-tf32 tensor cores, pre-passes included" % (M, N, K)}}
    else:  # gemm_streamed, gemm_streamed_f16
        M, N, K = (int(v) for v in args.gemm_shape.split(",")) if args.gemm_shape != "8192,8192,8192" else \
            (32768, 32768, 32768)
        f16 = op.endswith("f16")
        r = bench_gemm_streamed(ctx, args.steps, args.warmup, M, N, K, f16=f16)
        es = 2 if f16 else 4
        r.update(unit="TFLOP/s", roofline=roofline("tensor" if f16 else "tensor_3xtf32", r["value"], pk),
                 e2e={"value": round(r["value"], 3), "h2d": (M * K + K * N) * es, "d2h": M * N * es})
        extra = {"config": {"workload": "GEMM %dx%dx%d %s streamed from pinned host memory, B resident, %d row "
                                        "blocks in a two-slot ring" % (M, N, K, "f16" if f16 else "fp32",
                                                                       r["blocks"])},
                 "host_link_GBps": round(r["link_GBps"], 2)}
    if ctx.rank == 0:
        line = op_line(op, r)
        line.update({"metric": METRIC, "n_gpus": ctx.world, "steps": args.steps, "warmup": args.warmup,
                     "higher_is_better": True})
        line.update(extra)
        emit(line)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--op", default="all", choices=["all"] + SINGLE_OPS,
                    help="all = every op, headline f16 GEMM last; otherwise one op alone (profiling)")
    ap.add_argument("--gemm-shape", default="8192,8192,8192", help="M,N,K of the f16 GEMM")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline legs")
    ap.add_argument("--no-e2e", action="store_true", help="one op's device-resident timing only (profiling)")
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
    want_cpu = not args.no_cpu
    rows = {}  # the BASELINE rows' headline figures (one GPU)

    if rank == 0:
        emit({"peaks": {"hbm": [pk.get("hbm_gbs"), "GB/s", pk["source"] + " copy"],
                        "tensor": [pk.get("bf16_tflops"), "TFLOP/s", pk["source"] + " bf16 burst"],
                        "tensor_sustained": [pk.get("bf16_tflops_sustained"), "TFLOP/s", pk["source"]],
                        "tensor_3xtf32": [round(pk.get("bf16_tflops", FALLBACK["bf16_tflops"]) / 6.0, 2), "TFLOP/s",
                                          "bf16 burst / 6 (3 tf32 MMAs at half rate)"],
                        "fp32": [round(FP32_SIMT_TFLOPS, 1), "TFLOP/s", "nominal FFMA"]},
              "cpu_threads": cpu_threads()})
    if args.op == "all" and world == 1:
        one = Ctx(1, 0, local_rank)
        s = max(5, min(args.steps, 20))
        # widenings beyond the reference's dtype interval, and channelscale
        # (BASELINE runs it fused into the conv): printed first
        for op in ("softmax", "rmsnorm", "channelscale", "reduce"):
            r = bench_rowop_f16(one, op, s, 3)
            emit({"op": op + "_f16", "value": round(r["value"], 1), "unit": "GB/s", "ms": round(r["ms"], 5),
                  "roofline": {"bound": "hbm", "peak": pk["hbm_gbs"], "frac": round(r["value"] / pk["hbm_gbs"], 4)}})
        r = bench_conv_f16(one, max(3, s // 2), 3)
        tp = pk.get("bf16_tflops", FALLBACK["bf16_tflops"])
        emit({"op": "conv_f16", "value": round(r["value"], 2), "unit": "TFLOP/s", "ms": round(r["ms"], 5),
              "roofline": {"bound": "tensor", "peak": tp, "frac": round(r["value"] / tp, 4)}})
        r = bench_gemm_f32_tc(one, max(3, s // 2), 3)
        emit({"op": "gemm_f32_8192_3xtf32", "value": round(r["value"], 2), "unit": "TFLOP/s", "ms": round(r["ms"], 4),
              "roofline": {"bound": "tensor", "peak": round(tp / 6, 2), "frac": round(r["value"] / (tp / 6), 4)}})
        r = measure_rowop(one, "channelscale", s, 3, pk)
        emit(op_line("channelscale", r, cpu_rowop("channelscale", 8192, 16384) if want_cpu else None))
        torch.cuda.empty_cache()

        # the BASELINE rows, compact, last before the headline
        r = measure_gemm_f32(one, s, 3, pk)
        emit(summarize(rows, op_line("gemm_f32_512", r, cpu_gemm_f32() if want_cpu else None)))
        for op in ("reduce", "reduce_scalar", "rmsnorm", "softmax"):
            r = measure_rowop(one, op, s, 3, pk)
            cpu = (cpu_reduce_scalar() if op == "reduce_scalar" else cpu_rowop(op, 8192, 16384)) if want_cpu else None
            emit(summarize(rows, op_line(op, r, cpu)))
            torch.cuda.empty_cache()
        r = measure_conv(one, max(3, s // 2), 3, pk)
        emit(summarize(rows, op_line("conv_n32", r, cpu_conv(32, 256, 56, 56, 256, 1) if want_cpu else None)))
        torch.cuda.empty_cache()
        r = measure_decode(one, s, 3, pk)
        # the chain at every batch the decode config names (device-resident, GB/s)
        sweep = {}
        for b in (1, 2, 4, 8, 16):
            sweep[str(b)] = round(measure_decode(one, s, 3, pk, Bt=b, e2e=False)["value"], 1)
            torch.cuda.empty_cache()
        emit(summarize(rows, op_line("decode_b32", r, cpu_decode() if want_cpu else None, b_sweep_GBps=sweep)))
        torch.cuda.empty_cache()

    if args.op == "all" and world > 1:
        r = bench_conv_sharded(ctx, max(3, min(args.steps, 10)), 3)
        if rank == 0:
            emit({"op": "conv_n32_batch_sharded", "value": round(r["value"], 2), "unit": "TFLOP/s",
                  "ms": round(r["ms"], 4), "n_gpus": world, "parallelism": r["parallelism"], "scaling": "strong"})
        r = bench_decode_sharded(ctx, max(5, min(args.steps, 20)), 3)
        if rank == 0:
            emit({"op": "decode_b32_column_sharded", "value": round(r["value"], 1), "unit": "GB/s",
                  "ms": round(r["ms"], 4), "n_gpus": world, "parallelism": r["parallelism"], "scaling": "strong"})

    g = bench_gemm_f16(ctx, args.steps, args.warmup, M, N, K, profile_only=args.no_e2e)
    if args.no_e2e:
        if rank == 0:
            emit({"op": "gemm_f16", "value": round(g["value"], 3), "unit": "TFLOP/s", "ms": round(g["ms"], 5),
                  "kernel_ms": round(g["kernel_ms"], 5), "n_gpus": world, "steps": args.steps,
                  "config": {"M": M, "N": N, "K": K}, "note": "--no-e2e: timed steps only"})
        if world > 1:
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()
        return 0
    clocks = g["clocks"]
    if clocks:
        clocks.pop("samples", None)

    roof = roofline("tensor", g["kernel_tflops"], pk, traffic_for("gemm_f16_%dx%dx%d_n%d" % (M, N, K, world))) \
        if world == 1 else fused_roofline(g, M, N, K, world, pk)
    roof.pop("peak_source", None)  # in the peaks line
    line = {"metric": METRIC, "value": round(g["value"], 3), "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(g["ms"], 5), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f16", "data": "synthetic N(0,0.02)",
            "config": {"workload": "f16 GEMM %dx%dx%d (configs[3])" % (M, N, K), "M": M, "N": N, "K": K,
                       "parallelism": g["parallelism"] if world > 1 else "1 GPU", "l2": "inputs > L2"},
            "roofline": roof, "e2e": g["e2e"], "gpu_launches": g["launches"], "clocks": clocks,
            "sustained": g["sustained"], "check": g["check"]}
    if world == 1 and want_cpu:
        cb = cpu_gemm_f16(M, N, K, rows=gemm_f16_cpu_rows())
        line["cpu_baseline"] = {k: (round(v, 6) if isinstance(v, float) else v) for k, v in cb.items()
                                if k != "seconds"}
    if rank == 0:
        if rows:
            # every BASELINE row again in one short line, so that the rows and the
            # headline sit together in the last ~1.5 KB of the output
            emit({"baseline_rows": {"fields": ["value", "unit", "roofline_frac", "e2e", "cpu_baseline"], **rows}})
        emit(line)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
