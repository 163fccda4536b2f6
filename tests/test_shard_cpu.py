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
