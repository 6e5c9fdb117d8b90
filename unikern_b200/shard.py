"""Multi-GPU plumbing for the N-sharded f16 GEMM (one process per GPU).

The north star splits the columns of B and C over the GPUs of one node and
all-gathers C.  Here the all-gather is fused into the GEMM: every rank holds a
full C[M][N]; rank r computes its column block and its kernel stores each
tile into its own C and into every peer's C (CUDA IPC mappings over NVLink).
torch.distributed is the plumbing: it carries the IPC handles once, and an
all-reduce of one float after each GEMM is the stream-ordered barrier that
tells every rank its C is complete.
"""
from __future__ import annotations

import ctypes as C

from . import abi

MAX_RANKS = 8  # the kernel stores to at most 8 copies of C


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
        self.flag = torch.zeros(1, device="cuda")
        self.launches_per_step = 1  # this library's kernels per step (the barrier is NCCL's)

    def describe(self):
        return "N-sharded over %d GPUs (%d columns each), all-gather fused into the GEMM epilogue " \
               "(peer stores over NVLink) + NCCL barrier" % (self.world, self.n1 - self.n0)

    def b_shard(self, B):
        return B[:, self.n0:self.n1]

    def launch(self, A, B_shard, stream=None):
        """This rank's GEMM: its column block, stored into every rank's C."""
        abi.check(abi.lib().uk_cuda_gemm_f16_allgather(
            A.data_ptr(), A.stride(0), B_shard.data_ptr(), B_shard.stride(0), self.c_list, self.world, self.ldc,
            self.M, self.n1 - self.n0, self.K, self.n0, abi._stream(stream)))

    def barrier(self):
        """Stream-ordered: after it, every rank's stores into this rank's C are done."""
        import torch.distributed as dist
        dist.all_reduce(self.flag, group=self.group)

    def run(self, A, B_shard, C_full, stream=None):
        self.launch(A, B_shard, stream)
        self.barrier()

    def close(self):
        self.peers.close()
