"""Multi-GPU plumbing for the N-sharded f16 GEMM (one process per GPU).

The north star splits the columns of B and C over the GPUs of one node and
all-gathers C.  Here the all-gather is fused into the GEMM: every rank holds a
full C[M][N]; rank r computes its column block and its kernel stores each
tile into its own C and into every peer's C (CUDA IPC mappings over NVLink).
torch.distributed is the plumbing: it carries the IPC handles once.  After
each GEMM a device-side barrier (flags posted into every rank's memory over
NVLink, waited for with a time limit) tells every rank its C is complete.
"""
from __future__ import annotations

import ctypes as C
import os

from . import abi

MAX_RANKS = 8  # the kernel stores to at most 8 copies of C
_CUDART = None
CUDA_MEMCPY_DEFAULT = 4
CUDA_HOST_REGISTER_PORTABLE = 1


def cudart():
    """The CUDA runtime torch loaded (for stream-ordered strided host copies
    of the host-to-host sharded path; the library's own entry points link a
    static runtime and are not involved)."""
    global _CUDART
    if _CUDART is None:
        import torch  # noqa: F401  (loads libcudart.so.12 into the process)
        lib = C.CDLL("libcudart.so.12")
        lib.cudaMemcpy2DAsync.restype = C.c_int
        lib.cudaMemcpy2DAsync.argtypes = [C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t, C.c_size_t, C.c_size_t,
                                          C.c_int, C.c_void_p]
        lib.cudaHostRegister.restype = C.c_int
        lib.cudaHostRegister.argtypes = [C.c_void_p, C.c_size_t, C.c_uint]
        lib.cudaHostUnregister.restype = C.c_int
        lib.cudaHostUnregister.argtypes = [C.c_void_p]
        _CUDART = lib
    return _CUDART


def copy2d(dst, dpitch, src, spitch, width, height, stream):
    """height rows of `width` bytes, stream-ordered (cudaMemcpyDefault: either
    side may be host or device memory)."""
    rc = cudart().cudaMemcpy2DAsync(dst, dpitch, src, spitch, width, height, CUDA_MEMCPY_DEFAULT, stream)
    if rc != 0:
        raise RuntimeError("cudaMemcpy2DAsync failed with CUDA error %d" % rc)


def column_split(N: int, world: int, rank: int, align: int = 8):
    """[n0, n1): the contiguous block of C's columns owned by `rank`.

    Blocks are multiples of `align` columns (16-byte f16 stores) and as even
    as possible; the last rank takes the remainder."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank %d of %d" % (rank, world))
    units = (N + align - 1) // align
    per, extra = divmod(units, world)
    u0 = rank * per + min(rank, extra)
    u1 = u0 + per + (1 if rank < extra else 0)
    return min(N, u0 * align), min(N, u1 * align)


def store_order(world: int, rank: int):
    """Ranks whose C a tile is written to, local first then around the ring,
    so that no GPU receives every rank's first store at once."""
    return [(rank + i) % world for i in range(world)]


def gather_objects(obj, group=None):
    import torch.distributed as dist
    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, obj, group=group)
    return out


class PeerLost(RuntimeError):
    """A peer rank left or stopped stepping: the runner's exit code 4."""

    code = 4


class PeerWatch:
    """Host-side liveness of the ranks between steps.

    Before a step's GPU work, every rank posts "step n" to the process
    group's key-value store and waits, for at most `timeout_s`, until every
    peer has posted the same step.  A peer that exited, crashed or stopped
    stepping is found here, on the host and before this rank launches a
    kernel that stores into that peer's memory, and the wait ends with
    PeerLost naming the missing ranks: an error status, never a hang (the
    reference's runner, likewise, ends a failed run with an exit code,
    src/main.cpp:469-539).  Keys of finished steps are removed as the ranks
    move on."""

    def __init__(self, timeout_s: float = 5.0, group=None, prefix: str = "uk_hb"):
        import torch.distributed as dist
        from torch.distributed import distributed_c10d as c10d
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.store = c10d._get_default_store()
        self.timeout_s = timeout_s
        self.prefix = prefix
        self.n = 0

    def _key(self, step, rank):
        return "%s/%d/%d" % (self.prefix, step, rank)

    def step(self):
        """Post this rank's next step and wait for every peer's; returns the
        step number, raises PeerLost when a peer does not post in time."""
        import datetime
        n = self.n
        self.store.set(self._key(n, self.rank), b"1")
        keys = [self._key(n, r) for r in range(self.world) if r != self.rank]
        try:
            if keys:
                self.store.wait(keys, datetime.timedelta(seconds=self.timeout_s))
        except Exception as e:  # the store's timeout, or its server (rank 0) gone
            missing = []
            for r in range(self.world):
                if r == self.rank:
                    continue
                try:
                    if not self.store.check([self._key(n, r)]):
                        missing.append(r)
                except Exception:
                    missing.append(r)
            raise PeerLost("step %d: rank(s) %s did not reach the step within %.1f s (%s)"
                           % (n, missing or "?", self.timeout_s, type(e).__name__)) from None
        if n >= 2:  # every peer has posted step n, so all are past step n - 2
            try:
                self.store.delete_key(self._key(n - 2, self.rank))
            except Exception:
                pass
        self.n = n + 1
        return n


class PeerBuffers:
    """Device pointers of every rank's copy of one buffer (peers via CUDA IPC)."""

    def __init__(self, local, group=None):
        import torch.distributed as dist
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        lib = abi.lib()
        hs = lib.uk_cuda_ipc_handle_size()
        h = (C.c_char * hs)()
        off = C.c_uint64()
        abi.check(lib.uk_cuda_ipc_export(local.data_ptr(), h, C.byref(off)))
        handles = gather_objects((bytes(h), off.value), group)
        self.ptrs, self._opened = [], []
        for r, (hb, o) in enumerate(handles):
            if r == self.rank:
                self.ptrs.append(local.data_ptr())
                continue
            p = C.c_void_p()
            abi.check(lib.uk_cuda_ipc_import(C.create_string_buffer(hb, len(hb)), o, C.byref(p)))
            self.ptrs.append(p.value)
            self._opened.append((p.value, o))

    def close(self):
        for p, o in self._opened:
            abi.lib().uk_cuda_ipc_close(p, o)
        self._opened = []


class DeviceBarrier:
    """Stream-ordered barrier of the ranks on the GPUs themselves
    (uk_cuda_peer_barrier): each rank's flag array (one unsigned per rank) is
    opened by every peer once; a step posts an ever-growing epoch into every
    rank's array and waits, bounded by timeout_s, for every rank's post in its
    own.  It replaces a one-float NCCL all-reduce (about 25 us on 8 GPUs) after
    the sharded kernels; UK_BARRIER=nccl keeps the all-reduce.  A wait that
    runs out sets bit 32 of uk_cuda_pipeline_fault."""

    def __init__(self, group=None, timeout_s: float = 2.0):
        import torch
        import torch.distributed as dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.kind = "nccl" if os.environ.get("UK_BARRIER", "device") == "nccl" else "device"
        self.timeout_ns = int(timeout_s * 1e9)
        self.epoch = 0
        self.flag = torch.zeros(1, device="cuda")
        self.peers = None
        if self.kind == "device" and self.world > 1:
            self.flags = torch.zeros(MAX_RANKS, dtype=torch.int32, device="cuda")
            self.peers = PeerBuffers(self.flags, group)
            self.ptrs = (C.c_void_p * self.world)(*self.peers.ptrs)

    def __call__(self, stream=None):
        import torch.distributed as dist
        if self.world == 1:
            return
        if self.kind == "nccl":
            dist.all_reduce(self.flag, group=self.group)
            return
        self.epoch += 1
        abi.check(abi.lib().uk_cuda_peer_barrier(self.ptrs, self.world, self.rank, self.epoch & 0xFFFFFFFF,
                                                 self.timeout_ns, abi._stream(stream)))

    def close(self):
        if self.peers is not None:
            import torch
            torch.cuda.synchronize()
            self.peers.close()
            self.peers = None


class GemmAllGather:
    """C = A * B on `world` GPUs: B and C split by columns, C all-gathered."""

    def __init__(self, C_full, M: int, N: int, K: int, group=None):
        import torch
        import torch.distributed as dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > MAX_RANKS:
            raise ValueError("the fused all-gather stores to at most %d GPUs" % MAX_RANKS)
        self.M, self.N, self.K = M, N, K
        self.n0, self.n1 = column_split(N, self.world, self.rank)
        self.peers = PeerBuffers(C_full, group)
        order = store_order(self.world, self.rank)
        self.c_list = (C.c_void_p * self.world)(*[self.peers.ptrs[r] for r in order])
        self.ldc = C_full.stride(0)
        self.c_tensor, self.c_local = C_full, C_full.data_ptr()
        self.sync = DeviceBarrier(group)
        # this library's kernels per step: the GEMM, and the device barrier
        self.launches_per_step = 2 if self.sync.kind == "device" else 1

    def describe(self):
        return "N-sharded over %d GPUs (%d columns each), all-gather fused into the GEMM epilogue " \
               "(peer stores over NVLink) + %s barrier" % (self.world, self.n1 - self.n0, self.sync.kind)

    def b_shard(self, B):
        return B[:, self.n0:self.n1]

    def launch(self, A, B_shard, stream=None):
        """This rank's GEMM: its column block, stored into every rank's C."""
        abi.check(abi.lib().uk_cuda_gemm_f16_allgather(
            A.data_ptr(), A.stride(0), B_shard.data_ptr(), B_shard.stride(0), self.c_list, self.world, self.ldc,
            self.M, self.n1 - self.n0, self.K, self.n0, abi._stream(stream)))

    def barrier(self, stream=None):
        """Stream-ordered: after it, every rank's stores into this rank's C are done."""
        self.sync(stream)

    def run(self, A, B_shard, C_full, stream=None, watch=None):
        """One step; with a PeerWatch, every peer is confirmed alive on the
        host before the kernel stores into its C."""
        if watch is not None:
            watch.step()
        self.launch(A, B_shard, stream)
        self.barrier(stream)

    def close(self):
        self.sync.close()
        self.peers.close()


class HostGemmF16:
    """The N-sharded f16 GEMM from and to host memory, as a user of a node's
    GPUs calls it: A[M][K] and B[K][N] in, C[M][N] out, one host copy of each
    shared by the ranks (files in /dev/shm mapped by every rank and
    registered as page-locked memory; private pinned copies where /dev/shm is
    too small).  Each step, on the launching stream:

    1. rank r uploads its row block of A and its column block of B (a strided
       2-D copy) over its own host link, so every host byte crosses the host
       links once per step instead of once per rank;
    2. an NCCL all-gather over NVLink replicates A (its row blocks are
       contiguous);
    3. the GEMM with the fused all-gather of C (GemmAllGather.run);
    4. rank r downloads only its column block of C (a strided 2-D copy) into
       the shared host C.
    """

    def __init__(self, plan, A_src, B_src):
        import torch
        import torch.distributed as dist
        self.plan = plan
        M, N, K = plan.M, plan.N, plan.K
        w, r = plan.world, plan.rank
        self.split_a = M % w == 0
        self.r0, self.r1 = (M // w * r, M // w * (r + 1)) if self.split_a else (0, M)
        self.n0, self.n1 = plan.n0, plan.n1
        need = (M * K + K * N + M * N) * 2
        st = os.statvfs("/dev/shm") if os.path.isdir("/dev/shm") else None
        ok = st is not None and st.f_bavail * st.f_frsize > 2 * need
        self.shared = bool(gather_objects(ok, plan.group) == [True] * w)
        self.paths = []
        if self.shared:
            tag = "uk_e2e_%s_%d_%dx%dx%d" % (os.environ.get("MASTER_PORT", "0"), os.getppid(), M, N, K)
            bufs = []
            for name, n in (("A", M * K), ("B", K * N), ("C", M * N)):
                path = "/dev/shm/%s_%s" % (tag, name)
                self.paths.append(path)
                if r == 0:
                    t = torch.from_file(path, shared=True, size=n, dtype=torch.float16)
                dist.barrier(group=plan.group)
                if r != 0:
                    t = torch.from_file(path, shared=True, size=n, dtype=torch.float16)
                bufs.append(t)
            self.Ah, self.Bh, self.Ch = bufs[0].view(M, K), bufs[1].view(K, N), bufs[2].view(M, N)
            if r == 0:
                self.Ah.copy_(A_src.cpu())
                self.Bh.copy_(B_src.cpu())
            for t in (self.Ah, self.Bh, self.Ch):
                rc = cudart().cudaHostRegister(t.data_ptr(), t.numel() * 2, CUDA_HOST_REGISTER_PORTABLE)
                if rc != 0:
                    raise RuntimeError("cudaHostRegister failed with CUDA error %d" % rc)
            dist.barrier(group=plan.group)
        else:
            self.Ah = A_src.cpu().pin_memory()
            self.Bh = B_src.cpu().pin_memory()
            self.Ch = torch.empty((M, N), dtype=torch.float16).pin_memory()
        self.Ad = torch.empty((M, K), dtype=torch.float16, device="cuda")
        self.Bd = torch.empty((K, self.n1 - self.n0), dtype=torch.float16, device="cuda")
        # whole-job bytes per step (the sum over the ranks' links)
        self.h2d_bytes = (M * K if self.split_a else w * M * K) * 2 + K * N * 2
        self.d2h_bytes = M * N * 2

    def step(self, stream=None):
        import torch
        import torch.distributed as dist
        p = self.plan
        s = (stream or torch.cuda.current_stream()).cuda_stream
        M, N, K = p.M, p.N, p.K
        nb = self.n1 - self.n0
        rows = self.r1 - self.r0
        copy2d(self.Ad.data_ptr() + self.r0 * K * 2, K * 2, self.Ah.data_ptr() + self.r0 * K * 2, K * 2, K * 2,
               rows, s)
        copy2d(self.Bd.data_ptr(), nb * 2, self.Bh.data_ptr() + self.n0 * 2, N * 2, nb * 2, K, s)
        if self.split_a and p.world > 1:
            dist.all_gather_into_tensor(self.Ad, self.Ad[self.r0:self.r1], group=p.group)
        p.run(self.Ad, self.Bd, None)
        copy2d(self.Ch.data_ptr() + self.n0 * 2, N * 2, p.c_local + self.n0 * 2, p.ldc * 2, nb * 2, M, s)

    def check_host(self, step_fn=None):
        """After one step: the host C against this rank's device C (the full
        gathered C): max |difference| over the rank's view of the host C (all
        of it when shared, its own block otherwise), max over ranks."""
        import torch
        import torch.distributed as dist
        (step_fn or self.step)()
        torch.cuda.synchronize()
        dist.barrier(group=self.plan.group)
        dev = self.plan.c_tensor.cpu()
        cols = slice(None) if self.shared else slice(self.n0, self.n1)
        d = float((dev[:, cols].float() - self.Ch[:, cols].float()).abs().max().item())
        t = torch.tensor([d], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.plan.group)
        return {"max_abs_diff_host_vs_device": float(t.item()), "host_c": "shared" if self.shared else "per rank"}

    def close(self):
        import torch.distributed as dist
        torch_sync()
        if self.shared:
            for t in (self.Ah, self.Bh, self.Ch):
                cudart().cudaHostUnregister(t.data_ptr())
            dist.barrier(group=self.plan.group)
            if self.plan.rank == 0:
                for path in self.paths:
                    try:
                        os.unlink(path)
                    except OSError:
                        pass


def torch_sync():
    import torch
    torch.cuda.synchronize()


def batch_split(N: int, world: int, rank: int):
    """[b0, b1): the contiguous block of images owned by `rank` (as even as
    possible; the first N % world ranks take one more)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank %d of %d" % (rank, world))
    per, extra = divmod(N, world)
    b0 = rank * per + min(rank, extra)
    return b0, b0 + per + (1 if rank < extra else 0)


class ConvBatchShard:
    """conv2d (NCHW, stride 1, zero padding, fused per-channel scale) over
    `world` GPUs: the batch is split into contiguous image blocks, weights and
    scale are replicated, and the output is all-gathered so every rank holds
    the full Y[N][Oc][Ho][Wo].  Images are independent, so the only exchange is
    the gather.  On the tensor-core path it is fused into the conv's store:
    each rank's kernel writes its image block into every rank's Y (CUDA IPC
    mappings over NVLink, opened on the first run) and a barrier (UK_BARRIER)
    orders the ranks, so the exchange overlaps the compute tile by tile.
    Otherwise (and with UK_CONV_GATHER=nccl) an NCCL all-gather after the conv:
    in place into Y when the blocks are equal, through a padded staging buffer
    otherwise."""

    def __init__(self, N, Cc, H, W, Oc, Kh, Kw, pad, group=None):
        import torch.distributed as dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.N, self.C, self.H, self.W, self.Oc, self.Kh, self.Kw, self.pad = N, Cc, H, W, Oc, Kh, Kw, pad
        self.Ho, self.Wo = H + 2 * pad - Kh + 1, W + 2 * pad - Kw + 1
        self.blocks = [batch_split(N, self.world, r) for r in range(self.world)]
        self.b0, self.b1 = self.blocks[self.rank]
        self.even = len({b1 - b0 for b0, b1 in self.blocks}) == 1
        self._stage = None
        # the tensor-core kernel's workspace for this rank's images (None when
        # the shape runs the FFMA kernel)
        self.ws = abi.conv2d_workspace(max(1, self.b1 - self.b0), H, W, Cc, Kh, Kw, Oc, pad, abi.UK_CONV_NCHW) \
            if self.b1 > self.b0 else None
        self.fused = self.world > 1 and self.ws is not None and os.environ.get("UK_CONV_GATHER", "fused") != "nccl"
        self._peers = None
        self._ylist = None
        self.sync = DeviceBarrier(group) if self.fused else None
        # the hi/lo pre-passes and the conv (and the device barrier when fused)
        self.launches_per_step = 4 if self.fused else 3

    def describe(self):
        return "batch-sharded over %d GPUs (%d images each), %s" % (
            self.world, self.b1 - self.b0,
            "all-gather fused into the conv's store (peer stores over NVLink) + device barrier" if self.fused else
            "NCCL all-gather of Y")

    def _bind(self, Y):
        """Open every rank's Y once (a collective: every rank binds together)."""
        if self._peers is not None:
            if Y.data_ptr() != self._bound:
                raise ValueError("ConvBatchShard: the fused gather is bound to one Y buffer")
            return
        self._peers = PeerBuffers(Y, self.group)
        self._bound = Y.data_ptr()
        off = self.b0 * self.Oc * self.Ho * self.Wo * Y.element_size()
        order = store_order(self.world, self.rank)
        self._ylist = (C.c_void_p * self.world)(*[self._peers.ptrs[r] + off for r in order])

    def x_shard(self, X):
        return X[self.b0:self.b1]

    def launch(self, x_shard, Wt, Y, scale=None, stream=None):
        """This rank's images into its block of Y (and, fused, every rank's)."""
        n = self.b1 - self.b0
        if self.fused:
            self._bind(Y)
            ws = self.ws
            abi.check(abi.lib().uk_cuda_conv2d_f32_allgather(
                x_shard.data_ptr(), Wt.data_ptr(), self._ylist, self.world, n, self.H, self.W, self.C, self.Kh,
                self.Kw, self.Oc, self.pad, None if scale is None else scale.data_ptr(), ws.data_ptr(),
                ws.numel() * ws.element_size(), abi._stream(stream)))
            return
        if n:
            abi.conv2d_tc(x_shard, Wt, Y[self.b0:self.b1], n, self.H, self.W, self.C, self.Kh, self.Kw, self.Oc,
                          self.pad, scale, abi.UK_CONV_NCHW, self.ws, stream)

    def gather(self, Y, stream=None):
        """Every rank's block into every rank's Y."""
        import torch
        import torch.distributed as dist
        if self.world == 1:
            return
        if self.fused:  # the blocks were stored by the conv itself: order the ranks
            self.sync(stream)
            return
        def gather_into(out, mine):
            # NCCL gathers in place (the input is this rank's slot of the
            # output); gloo, used by the CPU tests, takes a list and a copy
            if out.is_cuda:
                dist.all_gather_into_tensor(out, mine, group=self.group)
            else:
                dist.all_gather(list(out.split(mine.shape[0])), mine.clone(), group=self.group)

        if self.even:
            gather_into(Y, Y[self.b0:self.b1])
            return
        mx = max(b1 - b0 for b0, b1 in self.blocks)
        if self._stage is None:
            self._stage = torch.empty((self.world * mx,) + tuple(Y.shape[1:]), dtype=Y.dtype, device=Y.device)
        mine = self._stage[self.rank * mx:(self.rank + 1) * mx]
        mine[: self.b1 - self.b0].copy_(Y[self.b0:self.b1])
        gather_into(self._stage, mine)
        for r, (b0, b1) in enumerate(self.blocks):
            if r != self.rank and b1 > b0:
                Y[b0:b1].copy_(self._stage[r * mx:r * mx + b1 - b0])

    def run(self, x_shard, Wt, Y, scale=None, stream=None):
        self.launch(x_shard, Wt, Y, scale, stream)
        self.gather(Y, stream)

    def close(self):
        if self.sync is not None:
            self.sync.close()
        if self._peers is not None:
            self._peers.close()
            self._peers = None


class DecodeColumnShard:
    """The decode layer's RMSNorm -> f16 GEMM over `world` GPUs: the weight's
    columns are split (W[:, n0:n1] on each rank, 14336 / 8 = 1792 for
    Llama-3-8B), the token rows and gamma are replicated, and every rank's
    kernel stores its column block of Y into all ranks' Y (peer stores over
    NVLink), so the all-gather is fused into the GEMM's store."""

    def __init__(self, Y_full, B: int, N: int, K: int, group=None):
        import torch.distributed as dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > MAX_RANKS:
            raise ValueError("the fused all-gather stores to at most %d GPUs" % MAX_RANKS)
        self.B, self.N, self.K = B, N, K
        self.n0, self.n1 = column_split(N, self.world, self.rank)
        self.peers = PeerBuffers(Y_full, group)
        order = store_order(self.world, self.rank)
        self.y_list = (C.c_void_p * self.world)(*[self.peers.ptrs[r] for r in order])
        self.ldy = Y_full.stride(0)
        self.ws = abi.decode_workspace(B, K)
        self.sync = DeviceBarrier(group)
        # the norm kernel and the GEMM, and the device barrier
        self.launches_per_step = 3 if self.sync.kind == "device" else 2

    def describe(self):
        return "weight columns sharded over %d GPUs (%d each), all-gather fused into the store" % (
            self.world, self.n1 - self.n0)

    def w_shard(self, W):
        return W[:, self.n0:self.n1]

    def launch(self, X, gamma, W_shard, eps=1e-5, stream=None):
        abi.check(abi.lib().uk_cuda_decode_rmsnorm_gemm_f16(
            X.data_ptr(), gamma.data_ptr(), eps, W_shard.data_ptr(), W_shard.stride(0), self.y_list, self.world,
            self.ldy, self.B, self.n1 - self.n0, self.K, self.n0, self.ws.data_ptr(),
            self.ws.numel() * self.ws.element_size(), abi._stream(stream)))

    def barrier(self, stream=None):
        self.sync(stream)

    def run(self, X, gamma, W_shard, eps=1e-5, stream=None):
        self.launch(X, gamma, W_shard, eps, stream)
        self.barrier(stream)

    def close(self):
        self.sync.close()
        self.peers.close()
