"""Row sharding host logic on the CPU: shard ranges and the all-gather of
output slices across ranks, with two gloo processes (no GPU). The per-rank
slice here is computed with a plain matmul over the rank's rows; on a B200
it is the fused decode + GEMV of the rank's row shard."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from drinkme_b200 import shard


def test_row_range_covers_every_row_once():
    for R in (1, 7, 16, 100, 1024, 8192, 25600, 151936):
        for world in (1, 2, 3, 4, 8):
            seen = []
            for rank in range(world):
                r0, r1 = shard.row_range(R, rank, world)
                assert 0 <= r0 <= r1 <= R
                assert (r1 - r0) % 16 == 0 or r1 == R
                seen.extend(range(r0, r1))
            assert seen == list(range(R)), (R, world)
    with pytest.raises(ValueError):
        shard.row_range(10, 2, 2)


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, R, C, M, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(0)
        W = torch.randn(R, C, generator=g)
        x = torch.randn(M, C, generator=g)
        r0, r1 = shard.row_range(R, rank, world)
        local = x @ W[r0:r1].T
        full = shard.gather_rows(local, R, world)
        ok = torch.allclose(full, x @ W.T, atol=1e-5, rtol=1e-5)
        q.put((rank, bool(ok), tuple(full.shape)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("R,M", [(64, 1), (100, 3), (48, 8)])
def test_gather_rows_two_gloo_ranks(R, M):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, R, 32, M, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    got = sorted(q.get(timeout=10) for _ in range(2))
    assert got == [(0, True, (M, R)), (1, True, (M, R))]


def _exchange_worker(rank, world, port, leave, q):
    import datetime
    import time

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=6))
    if rank == leave:
        os._exit(0)  # this rank leaves before the handle exchange
    t0 = time.perf_counter()
    try:
        shard.exchange_handles(bytes([rank]) * 64, world)
        q.put((rank, "returned", time.perf_counter() - t0))
    except Exception as e:  # noqa: BLE001 - the survivor must raise, whatever the backend's type
        q.put((rank, type(e).__name__, time.perf_counter() - t0))
    os._exit(0)


def test_handle_exchange_raises_when_a_rank_left():
    """PeerGather's collective IPC-handle exchange over two gloo ranks, one of
    which exits before it: the survivor raises within the process group's
    timeout (6 s here) instead of waiting forever."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_exchange_worker, args=(r, 2, port, 1, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    rank, what, secs = q.get(timeout=10)
    assert rank == 0 and what != "returned", what
    assert secs < 6 + 10


def _exchange_ok_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q.put((rank, shard.exchange_handles(bytes([rank + 1]) * 64, world)))
    finally:
        dist.destroy_process_group()


def test_handle_exchange_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_exchange_ok_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    got = dict(q.get(timeout=10) for _ in range(2))
    assert got[0] == got[1] == [bytes([1]) * 64, bytes([2]) * 64]
