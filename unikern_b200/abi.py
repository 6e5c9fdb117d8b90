"""ctypes binding of include/unikern_cuda.h (the reference-side binding a
Python caller would add; the C++ caller links the library directly).

Wrappers take torch CUDA tensors only to obtain device pointers and the
current stream; every computation happens in libunikern_cuda.so.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import os

_LIB = None
# UNIKERN_CUDA_LIB names another build of the same library (same ABI)
_PATH = Path(os.environ.get("UNIKERN_CUDA_LIB") or Path(__file__).resolve().parent / "_lib" / "libunikern_cuda.so")

vp, i64, i32, f32, sz = C.c_void_p, C.c_int64, C.c_int, C.c_float, C.c_size_t

# name -> (restype, argtypes); must match include/unikern_cuda.h
PROTOTYPES = {
    "uk_cuda_last_error": (C.c_char_p, []),
    "uk_cuda_abi_version": (i32, []),
    "uk_cuda_device_supported": (i32, []),
    "uk_cuda_channelscale_f32": (i32, [vp, vp, vp, i64, i64, vp]),
    "uk_cuda_reduce_workspace_size": (sz, [i64, i64]),
    "uk_cuda_reduce_f32": (i32, [vp, vp, i64, i64, vp, sz, vp]),
    "uk_cuda_reduce_workspace_size_width": (sz, [i64, i64, i64]),
    "uk_cuda_reduce_f32_width": (i32, [vp, vp, i64, i64, i64, vp, sz, vp]),
    "uk_cuda_reduce_f16": (i32, [vp, vp, i64, i64, vp, sz, vp]),
    "uk_cuda_reduce_f16_width": (i32, [vp, vp, i64, i64, i64, vp, sz, vp]),
    "uk_cuda_reduce_f32_noalloc": (i32, [vp, vp, i64, i64, vp]),
    "uk_cuda_rmsnorm_f32": (i32, [vp, vp, vp, i64, i64, f32, vp]),
    "uk_cuda_softmax_f32": (i32, [vp, vp, i64, i64, vp]),
    "uk_cuda_gemm_f32": (i32, [vp, vp, vp, i32, i32, i32, vp]),
    "uk_cuda_gemm_f32_workspace_size": (sz, [i32, i32, i32]),
    "uk_cuda_gemm_f32_prefers_tc": (i32, [i32, i32, i32]),
    "uk_cuda_gemm_f32_ws": (i32, [vp, vp, vp, i32, i32, i32, vp, sz, vp]),
    "uk_cuda_gemm_f16": (i32, [vp, vp, vp, i32, i32, i32, vp]),
    "uk_cuda_gemm_f16_ld": (i32, [vp, i64, vp, i64, vp, i64, i32, i32, i32, vp]),
    "uk_cuda_conv2d_f32": (i32, [vp, vp, vp] + [i32] * 8 + [vp, i32, vp]),
    "uk_cuda_conv2d_workspace_size": (sz, [i32] * 9),
    "uk_cuda_conv2d_f32_ws": (i32, [vp, vp, vp] + [i32] * 8 + [vp, i32, vp, sz, vp]),
    "uk_cuda_conv2d_f32_allgather": (i32, [vp, vp, C.POINTER(vp), i32] + [i32] * 8 + [vp, vp, sz, vp]),
    "uk_cuda_pipeline_fault": (C.c_uint, []),
    "uk_cuda_selftest_wait": (i32, [i32, C.c_uint64, vp, vp]),
    "uk_cuda_gemm_f16_allgather": (i32, [vp, i64, vp, i64, C.POINTER(vp), i32, i64, i32, i32, i32, i64, vp]),
    "uk_cuda_peer_barrier": (i32, [C.POINTER(vp), i32, i32, C.c_uint, C.c_uint64, vp]),
    "uk_cuda_ipc_handle_size": (sz, []),
    "uk_cuda_ipc_export": (i32, [vp, vp, C.POINTER(C.c_uint64)]),
    "uk_cuda_ipc_import": (i32, [vp, C.c_uint64, C.POINTER(vp)]),
    "uk_cuda_ipc_close": (i32, [vp, C.c_uint64]),
    "uk_cuda_decode_workspace_size": (sz, [i32, i32]),
    "uk_cuda_decode_rmsnorm_gemm_f16": (i32, [vp, vp, f32, vp, i64, C.POINTER(vp), i32, i64, i32, i32, i32, i64,
                                               vp, sz, vp]),
    "uk_cuda_gemm_f16_host": (i32, [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, vp]),
    "uk_cuda_rowop_host": (i32, [i32, vp, vp, vp, vp, vp, vp, i64, i64, f32, i32, vp, sz, vp]),
    "uk_cuda_conv2d_f32_host_workspace_size": (sz, [i32] * 9),
    "uk_cuda_conv2d_f32_host": (i32, [vp, vp, vp, vp, vp, vp, vp, vp] + [i32] * 9 + [vp, sz, vp]),
    "uk_cuda_softmax_f16": (i32, [vp, vp, i64, i64, vp]),
    "uk_cuda_rmsnorm_f16": (i32, [vp, vp, vp, i64, i64, f32, vp]),
    "uk_cuda_channelscale_f16": (i32, [vp, vp, vp, i64, i64, vp]),
    "uk_cuda_conv2d_f16_workspace_size": (sz, [i32] * 9),
    "uk_cuda_conv2d_f16": (i32, [vp, vp, vp] + [i32] * 8 + [vp, i32, vp, sz, vp]),
    "uk_cuda_gemm_streamed_ring_size": (sz, [i32, i32, i32, i32, i32]),
    "uk_cuda_gemm_streamed": (i32, [vp, vp, vp, vp, vp, sz, i32, i32, i32, i32, i32, vp]),
    "uk_cuda_tile_plan": (i32, [i32, i32, C.POINTER(C.c_int64), i32, C.POINTER(C.c_int)]),
    "uk_cuda_solve_plan": (i32, [i32, i32, C.POINTER(C.c_int64), i32, i32, C.POINTER(C.c_int)]),
    "uk_cuda_last_launch": (i32, [C.POINTER(C.c_int)]),
    "uk_nccl_unique_id_size": (sz, []),
    "uk_nccl_get_unique_id": (i32, [vp]),
    "uk_nccl_comm_init": (i32, [vp, i32, i32, C.c_uint64, C.POINTER(vp)]),
    "uk_nccl_comm_destroy": (i32, [vp]),
    "uk_shard_gemm_f16_create": (i32, [vp, i32, i32, vp, i64, i32, i32, i32, C.c_uint64, C.POINTER(vp)]),
    "uk_shard_gemm_f16_columns": (i32, [vp, C.POINTER(C.c_int64), C.POINTER(C.c_int64)]),
    "uk_shard_gemm_f16_run": (i32, [vp, vp, i64, vp, i64, vp, C.c_uint64]),
    "uk_shard_gemm_f16_destroy": (i32, [vp]),
    "uk_kml_describe": (i32, [C.c_char_p, C.c_char_p, i32, C.c_char_p, sz]),
    "uk_run_kml": (i32, [C.c_char_p, C.c_char_p, C.c_char_p, i32, C.c_char_p, sz]),
    "uk_solve_kml": (i32, [C.c_char_p, C.c_char_p, C.c_char_p, i32, i32, C.c_char_p, sz]),
    "uk_run_cuda": (i32, [C.c_char_p, C.c_char_p, i32, i32, vp, C.c_char_p, sz]),
    "uk_calibrate": (i32, [C.c_char_p, C.c_char_p, i32, C.c_char_p, sz, C.c_char_p, sz]),
}

UK_CONV_KML, UK_CONV_NCHW = 0, 1
UK_OP = {"gemm": 0, "conv": 1, "reduce": 2, "softmax": 3, "rmsnorm": 4, "channelscale": 5}
SAMPLES = Path(__file__).resolve().parent / "samples"


class UkError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__("unikern_cuda error %d: %s" % (code, msg))
        self.code = code


def lib():
    """Load libunikern_cuda.so (raises if it was not built)."""
    global _LIB
    if _LIB is None:
        if not _PATH.exists():
            raise ImportError("libunikern_cuda.so not built: run `python -m unikern_b200.build` "
                              "(there is no CPU fallback)")
        l = C.CDLL(str(_PATH))
        for name, (res, args) in PROTOTYPES.items():
            fn = getattr(l, name)
            fn.restype, fn.argtypes = res, args
        _LIB = l
    return _LIB


def check(rc: int):
    if rc != 0:
        raise UkError(rc, lib().uk_cuda_last_error().decode())


def _stream(stream=None):
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def _p(t):
    return None if t is None else t.data_ptr()


# ---- torch-tensor wrappers (shapes follow the C ABI) -------------------------

def channelscale(X, S, Y, stream=None):
    L, Cc = X.shape
    check(lib().uk_cuda_channelscale_f32(_p(X), _p(S), _p(Y), L, Cc, _stream(stream)))


def reduce_workspace_size(rows, cols):
    return lib().uk_cuda_reduce_workspace_size(rows, cols)


def reduce(X, Y, workspace=None, stream=None):
    rows, cols = X.shape
    ws = workspace.numel() * workspace.element_size() if workspace is not None else 0
    check(lib().uk_cuda_reduce_f32(_p(X), _p(Y), rows, cols, _p(workspace), ws, _stream(stream)))


def reduce_width(X, Y, width, stream=None):
    """Row sums with the pass-1 width pinned (the UK_REDUCE_WIDTH knob);
    allocates its workspace through torch."""
    import torch
    rows, cols = X.shape
    n = lib().uk_cuda_reduce_workspace_size_width(rows, cols, width)
    ws = torch.empty(max(1, n), dtype=torch.uint8, device="cuda") if n else None
    check(lib().uk_cuda_reduce_f32_width(_p(X), _p(Y), rows, cols, width, _p(ws), n, _stream(stream)))


def reduce_f16(X, Y, width=0, stream=None):
    """Row sums of binary16 rows into binary16 Y (fp32 accumulation);
    width > 0 pins the pass-1 width.  Allocates its workspace through torch."""
    import torch
    rows, cols = X.shape
    n = (lib().uk_cuda_reduce_workspace_size_width(rows, cols, width) if width
         else lib().uk_cuda_reduce_workspace_size(rows, cols))
    ws = torch.empty(max(1, n), dtype=torch.uint8, device="cuda") if n else None
    if width:
        check(lib().uk_cuda_reduce_f16_width(_p(X), _p(Y), rows, cols, width, _p(ws), n, _stream(stream)))
    else:
        check(lib().uk_cuda_reduce_f16(_p(X), _p(Y), rows, cols, _p(ws), n, _stream(stream)))


def rmsnorm(X, W, Y, eps=1e-6, stream=None):
    L, Cc = X.shape
    check(lib().uk_cuda_rmsnorm_f32(_p(X), _p(W), _p(Y), L, Cc, eps, _stream(stream)))


def softmax(X, Y, stream=None):
    L, Cc = X.shape
    check(lib().uk_cuda_softmax_f32(_p(X), _p(Y), L, Cc, _stream(stream)))


def softmax_f16(X, Y, stream=None):
    L, Cc = X.shape
    check(lib().uk_cuda_softmax_f16(_p(X), _p(Y), L, Cc, _stream(stream)))


def rmsnorm_f16(X, W, Y, eps=1e-6, stream=None):
    L, Cc = X.shape
    check(lib().uk_cuda_rmsnorm_f16(_p(X), _p(W), _p(Y), L, Cc, eps, _stream(stream)))


def channelscale_f16(X, S, Y, stream=None):
    L, Cc = X.shape
    check(lib().uk_cuda_channelscale_f16(_p(X), _p(S), _p(Y), L, Cc, _stream(stream)))


def gemm_f32(A, B, Cm, stream=None):
    M, K = A.shape
    N = B.shape[1]
    check(lib().uk_cuda_gemm_f32(_p(A), _p(B), _p(Cm), M, N, K, _stream(stream)))


def gemm_f32_workspace(M, N, K):
    """The tensor-core f32 GEMM's workspace (a torch uint8 tensor), or None
    when the shape cannot take the tensor cores (K % 32 or N % 64 nonzero)."""
    import torch
    n = lib().uk_cuda_gemm_f32_workspace_size(M, N, K)
    return torch.empty(n, dtype=torch.uint8, device="cuda") if n else None


def gemm_f32_tc(A, B, Cm, workspace=None, stream=None):
    """C = A * B in fp32 on the tensor cores (split-tf32); allocates the
    workspace through torch when none is passed (FFMA when the shape has none)."""
    M, K = A.shape
    N = B.shape[1]
    ws = workspace if workspace is not None else gemm_f32_workspace(M, N, K)
    check(lib().uk_cuda_gemm_f32_ws(_p(A), _p(B), _p(Cm), M, N, K, _p(ws),
                                    0 if ws is None else ws.numel(), _stream(stream)))


def gemm_f16(A, B, Cm, stream=None):
    """A, B, C: torch.float16 (or int16/uint16 bit patterns) row-major, any strides
    with unit inner stride."""
    M, K = A.shape
    N = B.shape[1]
    check(lib().uk_cuda_gemm_f16_ld(_p(A), A.stride(0), _p(B), B.stride(0), _p(Cm), Cm.stride(0),
                                    M, N, K, _stream(stream)))


def conv2d(X, Wt, Y, N, H, W, Cc, Kh, Kw, Oc, pad=0, scale=None, layout=UK_CONV_NCHW, stream=None):
    check(lib().uk_cuda_conv2d_f32(_p(X), _p(Wt), _p(Y), N, H, W, Cc, Kh, Kw, Oc, pad, _p(scale), layout,
                                   _stream(stream)))


def decode_workspace(B, K):
    import torch
    n = lib().uk_cuda_decode_workspace_size(B, K)
    return torch.empty((max(n, 16) + 15) // 16 * 4, dtype=torch.float32, device="cuda")


def decode_rmsnorm_gemm(X, gamma, W, Y, eps=1e-5, workspace=None, stream=None):
    """Y[B][N] (f16) = f16(rmsnorm(X) * gamma) @ W (f16 [K][N])."""
    B, K = X.shape
    N = W.shape[1]
    ws = workspace if workspace is not None else decode_workspace(B, K)
    ys = (vp * 1)(Y.data_ptr())
    check(lib().uk_cuda_decode_rmsnorm_gemm_f16(_p(X), _p(gamma), eps, _p(W), W.stride(0), ys, 1, Y.stride(0), B, N,
                                                K, 0, _p(ws), ws.numel() * ws.element_size(), _stream(stream)))


def gemm_f16_host(Ah, Bh, Ch, Ad, Bd, Cd, chunks=0, stream=None):
    """C = A * B from pinned host tensors through device buffers, with the
    copies pipelined against the GEMM (row blocks of A and C)."""
    M, K = Ah.shape
    N = Bh.shape[1]
    check(lib().uk_cuda_gemm_f16_host(_p(Ah), _p(Bh), _p(Ch), _p(Ad), _p(Bd), _p(Cd), M, N, K, chunks,
                                      _stream(stream)))


def conv2d_host(Xh, Wh, Sh, Yh, Xd, Wd, Sd, Yd, N, H, W, Cc, Kh, Kw, Oc, pad=0, chunks=0, workspace=None,
                stream=None):
    """The fp32 NCHW conv from and to pinned host tensors through device
    buffers, image blocks pipelined (uploads, convs and downloads overlap).
    Allocates the workspace through torch when none is passed."""
    import torch
    if workspace is None:
        n = lib().uk_cuda_conv2d_f32_host_workspace_size(N, H, W, Cc, Kh, Kw, Oc, pad, chunks)
        workspace = torch.empty(((n + 15) // 16) * 4, dtype=torch.float32, device="cuda") if n else None
    nbytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
    check(lib().uk_cuda_conv2d_f32_host(_p(Xh), _p(Wh), _p(Sh), _p(Yh), _p(Xd), _p(Wd), _p(Sd), _p(Yd), N, H, W,
                                        Cc, Kh, Kw, Oc, pad, chunks, _p(workspace), nbytes, _stream(stream)))


def rowop_host(op, Xh, Wh, Yh, Xd, Wd, Yd, eps=1e-5, chunks=0, workspace=None, stream=None):
    """A row op from and to pinned host tensors through device buffers, the
    copies pipelined against the op over row blocks."""
    L, Cc = Xh.shape
    ws = workspace.numel() * workspace.element_size() if workspace is not None else 0
    check(lib().uk_cuda_rowop_host(UK_OP[op], _p(Xh), _p(Wh), _p(Yh), _p(Xd), _p(Wd), _p(Yd), L, Cc, eps, chunks,
                                   _p(workspace), ws, _stream(stream)))


def gemm_streamed(Ah, Bh, Ch, Bd, ring, block_rows, stream=None, ffma=False):
    """C = A * B (host tensors, f16 or fp32) with only B resident and A / C
    streamed through a two-slot device ring of block_rows-row blocks (fp32:
    the tensor cores where a block gains, unless ffma)."""
    import torch
    M, K = Ah.shape
    N = Bh.shape[1]
    kind = 1 if Ah.dtype == torch.float16 else (2 if ffma else 0)
    check(lib().uk_cuda_gemm_streamed(_p(Ah), _p(Bh), _p(Ch), _p(Bd), _p(ring), ring.numel() * ring.element_size(),
                                      M, N, K, kind, block_rows, _stream(stream)))


def gemm_streamed_ring(M, N, K, kind, block_rows):
    import torch
    n = lib().uk_cuda_gemm_streamed_ring_size(M, N, K, kind, block_rows)
    return torch.empty(n, dtype=torch.uint8, device="cuda")


def conv2d_workspace(N, H, W, Cc, Kh, Kw, Oc, pad=0, layout=UK_CONV_NCHW):
    import torch
    n = lib().uk_cuda_conv2d_workspace_size(N, H, W, Cc, Kh, Kw, Oc, pad, layout)
    return torch.empty(((n + 15) // 16) * 4, dtype=torch.float32, device="cuda") if n else None


def conv2d_tc(X, Wt, Y, N, H, W, Cc, Kh, Kw, Oc, pad=0, scale=None, layout=UK_CONV_NCHW, workspace=None,
              stream=None):
    """The tensor-core (split-tf32) convolution; allocates its workspace
    through torch when none is passed."""
    ws = workspace if workspace is not None else conv2d_workspace(N, H, W, Cc, Kh, Kw, Oc, pad, layout)
    nbytes = ws.numel() * ws.element_size() if ws is not None else 0
    check(lib().uk_cuda_conv2d_f32_ws(_p(X), _p(Wt), _p(Y), N, H, W, Cc, Kh, Kw, Oc, pad, _p(scale), layout,
                                      _p(ws), nbytes, _stream(stream)))


def conv2d_f16(X, Wt, Y, N, H, W, Cc, Kh, Kw, Oc, pad=0, scale=None, layout=UK_CONV_NCHW, workspace=None,
               stream=None):
    """fp16 convolution on the tensor cores (f16 tensors in and out)."""
    import torch
    n = lib().uk_cuda_conv2d_f16_workspace_size(N, H, W, Cc, Kh, Kw, Oc, pad, layout)
    ws = workspace
    if ws is None and n:
        ws = torch.empty(((n + 15) // 16) * 4, dtype=torch.float32, device="cuda")
    nbytes = ws.numel() * ws.element_size() if ws is not None else 0
    check(lib().uk_cuda_conv2d_f16(_p(X), _p(Wt), _p(Y), N, H, W, Cc, Kh, Kw, Oc, pad, _p(scale), layout,
                                   _p(ws), nbytes, _stream(stream)))


# ---- KML runner (host side) -----------------------------------------------------

def tile_plan(op: str, dims, f16: bool = False, sms: int = 0):
    """(tile_m, tile_n, k_block, stages) the library launches for a KML op."""
    d = (C.c_int64 * 6)(*(list(dims) + [0] * (6 - len(dims))))
    out = (C.c_int * 4)()
    check(lib().uk_cuda_tile_plan(UK_OP[op], int(f16), d, sms, out))
    return tuple(out)


FAMILIES = {0: "ffma", 1: "tcgen05-1sm", 2: "tcgen05-2sm", 3: "tcgen05-2sm-3xtf32", 4: "ffma-conv",
            5: "tcgen05-2sm-conv", 6: "tcgen05-skinny", 7: "ffma-kgroups"}


def solve_plan(M: int, N: int, K: int, f16: bool = False, sms: int = 0, allow_tc: bool = True):
    """The GEMM solve: dict(family, tile, k_block, stages, k_split, feasible, ns)."""
    d = (C.c_int64 * 6)(M, N, K, 0, 0, 0)
    out = (C.c_int * 8)()
    check(lib().uk_cuda_solve_plan(UK_OP["gemm"], int(f16), d, sms, int(allow_tc), out))
    return {"family": FAMILIES.get(out[0], out[0]), "tile": (out[1], out[2]), "k_block": out[3], "stages": out[4],
            "k_split": out[5], "feasible": out[6], "ns": out[7]}


def last_launch():
    """The plan of the last GEMM this thread launched: dict(family, tile,
    stages, k_split)."""
    out = (C.c_int * 6)()
    check(lib().uk_cuda_last_launch(out))
    return {"family": FAMILIES.get(out[0], out[0]), "tile": (out[1], out[2]), "stages": out[4], "k_split": out[5]}


def kml_describe(kml_json: str, hcs_json: str | None = None, sms: int = 0):
    """The KML contract of one declaration as a dict (raises UkError with the
    reference's rejection text for an invalid declaration)."""
    buf = C.create_string_buffer(1 << 16)
    rc = lib().uk_kml_describe(kml_json.encode(), hcs_json.encode() if hcs_json else None, sms, buf, len(buf))
    text = buf.value.decode()
    if rc != 0:
        raise UkError(rc, text)
    head, _, export = text.partition("export=")
    d = dict(line.split("=", 1) for line in head.splitlines() if "=" in line)
    d["export"] = export
    return d


def run_kml(hcs_json: str, kml_json: str, ledger: str | None = None, write_ledger: bool = True):
    """The nvidia branch of `unikern run` (write_ledger) / `verify`: returns
    (exit code, transcript)."""
    buf = C.create_string_buffer(1 << 16)
    rc = lib().uk_run_kml(hcs_json.encode(), kml_json.encode(), ledger.encode() if ledger else None,
                          int(write_ledger), buf, len(buf))
    return rc, buf.value.decode()


class RunOutcome(C.Structure):
    """uk_run_outcome: the fields of the reference's RunOutcome."""
    _fields_ = [("built", i32), ("ran", i32), ("verified", i32), ("max_rel", C.c_double),
                ("measured_ms", C.c_double), ("kernel_ms", C.c_double), ("migrations", i32), ("checks", i32),
                ("vram_free", C.c_ulonglong), ("vram_total", C.c_ulonglong), ("exit_code", i32),
                ("stream_path", C.c_char * 16)]


def run_cuda(hcs_json: str, kml_json: str, tile_m: int = 0, tile_n: int = 0):
    """run_cuda of one tree (no ledger): returns (RunOutcome, log)."""
    o = RunOutcome()
    buf = C.create_string_buffer(1 << 16)
    rc = lib().uk_run_cuda(hcs_json.encode(), kml_json.encode(), tile_m, tile_n, C.byref(o), buf, len(buf))
    if rc != 0:
        raise UkError(rc, buf.value.decode())
    return o, buf.value.decode()


def solve_kml(hcs_json: str, kml_json: str, ledger: str | None = None, write_ledger: bool = True, sms: int = 0):
    """The nvidia branch of `unikern solve`: returns (exit code, transcript).
    No GPU needed."""
    buf = C.create_string_buffer(1 << 14)
    rc = lib().uk_solve_kml(hcs_json.encode(), kml_json.encode(), ledger.encode() if ledger else None,
                            int(write_ledger), sms, buf, len(buf))
    return rc, buf.value.decode()


def calibrate(hcs_json: str, ledger: str, allow_unified: bool = False):
    """`unikern calibrate`: returns (exit code, calibrated HCS JSON or "",
    report)."""
    hbuf, buf = C.create_string_buffer(1 << 14), C.create_string_buffer(1 << 16)
    rc = lib().uk_calibrate(hcs_json.encode(), ledger.encode(), int(allow_unified), hbuf, len(hbuf), buf, len(buf))
    return rc, hbuf.value.decode() if rc == 0 else "", buf.value.decode()


def result_tokens(transcript: str):
    """key=value tokens of the UNIKERN_RESULT line (parsed by name, as the
    reference's runner does)."""
    for line in transcript.splitlines():
        if line.startswith("UNIKERN_RESULT"):
            return dict(t.split("=", 1) for t in line.split()[1:] if "=" in t)
    return None
