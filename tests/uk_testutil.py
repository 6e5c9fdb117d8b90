"""Helpers shared by the GPU parity tests: device copies and the tolerance
gates.  Tolerances (written here once, used by every parity test):

* f32 paths: rel_err <= 1e-4 against the f64 oracle, with the floor
  tau = RMS(ref) for sums of signed terms (gemm, conv, reduce) and
  tau = 1e-30 for softmax / rmsnorm / channelscale (outputs are exact
  scalings or bounded away from zero).  A floor of 1e-3 * RMS(ref) is not
  passable by the reference's own sequential fp32 cpu_ref (K = 512 uniform
  inputs give ~1e-3 on that scale), so the sum floor is the output scale and
  every such test also checks that the reference's fp32 algorithm passes the
  same gate;
* f16 GEMM: rel_err <= 2e-2 against the f64 oracle of the half inputs;
* channelscale, shapes and indices: bit-exact.
"""
import numpy as np

F32_TOL = 1e-4
F16_TOL = 2e-2
SUM_TAU = 1.0


def torch():
    import torch as t
    assert t.cuda.is_available(), "GPU tests need a CUDA device"
    return t


def dev(a):
    t = torch()
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        return t.from_numpy(a.view(np.int16)).cuda().view(t.float16)
    return t.from_numpy(a).cuda()


def host(t_):
    import torch as t
    t.cuda.synchronize()
    if t_.dtype == t.float16:
        return t_.cpu().view(t.int16).numpy().view(np.uint16)
    return t_.cpu().numpy()


def empty(shape, dtype="f32"):
    t = torch()
    return t.empty(shape, dtype=t.float32 if dtype == "f32" else t.float16, device="cuda")
