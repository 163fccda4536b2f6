"""The fused NVLink output gather (dm_gemv_gather, shard.PeerGather).

On one GPU (world = 1) the whole path runs with this GPU as the only rank:
the outputs land in the gathered buffer, bitwise dm_gemv's, and the flag
protocol lets a chained launch wait for its predecessor. With two GPUs, two
processes (one per GPU) row-shard fused tensors, chain launches that wait on
each other's flags, and every rank's gathered outputs must equal the
single-GPU result bitwise (same kernel, same per-tile sums) — skipped where
fewer than two GPUs are visible. No kernel of one GPU waits on another
kernel of the same GPU.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from drinkme_b200 import codec, radix_ops, shard, swap
from oracle import oracle

pytestmark = pytest.mark.gpu


def _packs(seed):
    g = torch.Generator().manual_seed(seed)
    shapes = ((256, 4096), (64, 4096), (64, 4096))
    Ws = [(torch.randn(r, c, generator=g) * s).to(torch.bfloat16) for (r, c), s in zip(shapes, (0.02, 0.05, 1.0))]
    return Ws, [codec.pack_weight_radix(W, "sip") for W in Ws]


def test_gather_world1_matches_dm_gemv_and_chains():
    dev = torch.device("cuda", 0)
    Ws, packs = _packs(1)
    rt = swap.to_device_radix_fused(packs, dev)
    rt2 = swap.to_device_radix(packs[0], dev)
    x = torch.randn(3, 4096, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16).to(dev)
    plan = shard.PeerGather([rt["R"], rt2["R"]], 3, torch.bfloat16, 0, 1, dev)
    try:
        for step in range(3):
            plan.gemv(rt, x, 0, wait=1)
            plan.gemv(rt2, x, 1, wait=0)
        torch.cuda.synchronize()
        assert torch.equal(plan.output(0), radix_ops.gemv_mc_fused(rt, x, None, torch.bfloat16))
        assert torch.equal(plan.output(1), radix_ops.gemv_mc_fused(rt2, x, None, torch.bfloat16))
        bits = np.concatenate([codec.bits_of(W) for W in Ws])
        y64, bound = oracle.gemv_bound(x.float().cpu().numpy(), bits)
        assert np.all(np.abs(plan.output(0).float().cpu().numpy() - y64) <= bound + np.abs(y64) * 2 ** -8)
        assert rt["rx_handle"].device_error() == 0 and rt2["rx_handle"].device_error() == 0
    finally:
        plan.close()


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, q, use_chain=False):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    plan = None
    try:
        Ws, packs = _packs(1)
        ranges = [shard.row_range(W.shape[0], rank, world) for W in Ws]
        rt = swap.to_device_radix_fused(packs, dev, ranges)
        slot = sum(shard.shard_rows_padded(W.shape[0], world) for W in Ws)
        x = torch.randn(2, 4096, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16).to(dev)
        plan = shard.PeerGather([slot, slot], 2, torch.bfloat16, rank, world, dev)
        if use_chain:
            # both linears in one persistent launch per step, the same waits
            chain = plan.chain([(rt, x, 0, 1, None), (rt, x, 1, 0, None)])
            for step in range(4):
                chain.run()
            torch.cuda.synchronize()
            assert int(plan.launch_count(1)) == 4
            chain.close()
        else:
            for step in range(4):
                plan.gemv(rt, x, 0, wait=1)
                plan.gemv(rt, x, 1, wait=0)
        torch.cuda.synchronize()
        got = plan.output(1).cpu()
        err = rt["rx_handle"].device_error()
        q.put((rank, got, err))
    finally:
        if plan is not None:
            plan.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("use_chain", [False, True], ids=["per-linear", "chain"])
def test_gather_two_gpus_equals_one_gpu(use_chain):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q, use_chain)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted((q.get(timeout=300) for _ in range(world)), key=lambda t: t[0])
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    Ws, packs = _packs(1)
    dev = torch.device("cuda", 0)
    x = torch.randn(2, 4096, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16).to(dev)
    # rank r's slot holds its fused shard's outputs [q_r | k_r | v_r]: the same
    # fused shard computed on one GPU gives them bitwise (same tensor, kernel and split)
    for rank, got, err in res:
        assert err == 0, rank
        slot = got.shape[1] // world
        for r in range(world):
            ranges = [shard.row_range(W.shape[0], r, world) for W in Ws]
            y = radix_ops.gemv_mc_fused(swap.to_device_radix_fused(packs, dev, ranges), x, None, torch.bfloat16).cpu()
            assert torch.equal(got[:, r * slot: r * slot + y.shape[1]], y), (rank, r)


def test_gather_wait_that_never_completes_returns_with_an_error():
    """A wait whose flags never reach the wanted launch count (a peer that
    never published: here this rank's own count raised by hand) gives up after
    its poll limit, records kErrWaitPeer (4) and sets the abort word; the next
    wait then returns at once even with the library's own multi-second bound.
    The GPU stays usable: a plain GEMV afterwards is exact."""
    import time

    dev = torch.device("cuda", 0)
    Ws, packs = _packs(3)
    rt = swap.to_device_radix(packs[0], dev)
    x = torch.randn(1, 4096, generator=torch.Generator().manual_seed(4)).to(torch.bfloat16).to(dev)
    plan = shard.PeerGather([rt["R"], rt["R"]], 1, torch.bfloat16, 0, 1, dev)
    try:
        plan.gemv(rt, x, 0)  # linear 0 runs once: its flag and launch count are 1
        torch.cuda.synchronize()
        assert rt["rx_handle"].device_error() == 0 and int(plan.abort_word().item()) == 0
        plan.launch_count(0).fill_(5)  # wait for a launch that never happens
        t0 = time.perf_counter()
        plan.gemv(rt, x, 1, wait=0, wait_polls=1 << 12)
        torch.cuda.synchronize()
        assert rt["rx_handle"].device_error() == 4  # kErrWaitPeer
        assert int(plan.abort_word().item()) != 0
        plan.gemv(rt, x, 1, wait=0)  # default bound: 2^23 polls, but the abort word ends it
        torch.cuda.synchronize()
        assert time.perf_counter() - t0 < 2.0
        assert rt["rx_handle"].device_error() == 4
        y = radix_ops.gemv_mc_fused(rt, x, None, torch.float32)
        y64, bound = oracle.gemv_bound(x.float().cpu().numpy(), codec.bits_of(Ws[0]))
        assert np.all(np.abs(y.cpu().numpy() - y64) <= bound)
        assert rt["rx_handle"].device_error() == 0
    finally:
        plan.close()
