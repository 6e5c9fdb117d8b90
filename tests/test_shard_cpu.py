"""Host logic of the multi-GPU GEMM on CPU: the column split, the store
order and the handle exchange, run as world-size-2 gloo process groups."""
import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from unikern_b200 import shard


@pytest.mark.parametrize("N,world", [(8192, 1), (8192, 2), (8192, 8), (14336, 8), (1000, 3), (8, 4), (24, 5)])
def test_column_split_partitions_exactly(N, world):
    blocks = [shard.column_split(N, world, r) for r in range(world)]
    assert blocks[0][0] == 0 and blocks[-1][1] == N
    for (a0, a1), (b0, b1) in zip(blocks, blocks[1:]):
        assert a1 == b0
    for a0, a1 in blocks:
        assert a0 % 8 == 0 and a1 >= a0
        assert a1 % 8 == 0 or a1 == N
    sizes = [b - a for a, b in blocks]
    assert max(sizes) - min(sizes) <= 8


def test_store_order_local_first_ring():
    assert shard.store_order(4, 2) == [2, 3, 0, 1]
    for w in range(1, 9):
        for r in range(w):
            o = shard.store_order(w, r)
            assert o[0] == r and sorted(o) == list(range(w))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        got = shard.gather_objects((b"handle-%d" % rank, 16 * rank))
        blocks = shard.gather_objects(shard.column_split(8192, world, rank))
        q.put((rank, got, blocks))
    finally:
        dist.destroy_process_group()


def test_handle_exchange_gloo_world2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, got, blocks in results:
        assert got == [(b"handle-0", 0), (b"handle-1", 16)]
        assert blocks == [(0, 4096), (4096, 8192)]


@pytest.mark.parametrize("N,world", [(32, 1), (32, 2), (32, 8), (7, 3), (2, 4), (33, 8)])
def test_batch_split_partitions_exactly(N, world):
    blocks = [shard.batch_split(N, world, r) for r in range(world)]
    assert blocks[0][0] == 0 and blocks[-1][1] == N
    for (a0, a1), (b0, b1) in zip(blocks, blocks[1:]):
        assert a1 == b0
    sizes = [b - a for a, b in blocks]
    assert max(sizes) - min(sizes) <= 1


def _conv_worker(rank, world, port, N, q):
    import torch
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        plan = shard.ConvBatchShard(N, 4, 6, 6, 3, 3, 3, 1, None)
        Y = torch.full((N, 3, 6, 6), float("nan"))
        # stand-in for this rank's conv: its images carry their own index
        for b in range(plan.b0, plan.b1):
            Y[b] = b
        plan.gather(Y)
        q.put((rank, Y[:, 0, 0, 0].tolist()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("N", [8, 5])  # equal blocks (in place) and unequal (staging)
def test_conv_batch_gather_gloo_world2(N):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_conv_worker, args=(r, 2, port, N, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, col in results:
        assert col == [float(b) for b in range(N)]


# ---- failure detection: a rank that leaves or stalls between steps ------------------

def _watch_worker(rank, world, port, mode, q):
    import time

    def report_and_exit(msg):
        # the queue's feeder thread must flush before the process ends abruptly
        q.put(msg)
        q.close()
        q.join_thread()
        os._exit(0)

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    watch = shard.PeerWatch(timeout_s=3.0)
    # every rank enters the watched steps together: on a cold machine one
    # rank's first imports can otherwise trail the others by seconds
    dist.barrier()
    done = []
    for step in range(4):
        if rank == world - 1 and step == 2:
            if mode == "leave":  # between steps, with no collective in flight
                report_and_exit((rank, "left", done))
            time.sleep(8.0)  # "stall": past the peers' limit
        t0 = time.monotonic()
        try:
            watch.step()
        except shard.PeerLost as e:
            report_and_exit((rank, "lost", done + [(step, str(e), time.monotonic() - t0)]))
        done.append(step)
    report_and_exit((rank, "ok", done))


@pytest.mark.parametrize("mode", ["leave", "stall"])
def test_peer_watch_reports_a_missing_rank_within_its_limit(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    world = 3
    procs = [ctx.Process(target=_watch_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        rank, what, info = q.get(timeout=120)
        res[rank] = (what, info)
    for p in procs:
        p.join(timeout=60)
    # the ranks that stayed all stop at step 2 with PeerLost, naming rank 2,
    # within about their 3 s limit -- none hangs
    for r in (0, 1):
        what, info = res[r]
        assert what == "lost", res
        step, msg, waited = info[-1]
        assert step == 2 and "[2]" in msg and waited < 15.0, info
        assert info[:-1] == [0, 1]
    assert res[2][0] in ("left", "lost", "ok")
