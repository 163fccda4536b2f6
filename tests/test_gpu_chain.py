"""A chain: several row-sharded linears in one persistent launch
(dm_chain_create / dm_chain_run, shard.PeerGather.chain) on one GPU.

Every link's output must be bitwise the per-linear call's (dm_gemv through
radix_ops) on the same activations, whether the link reads a fixed input or
an earlier link's output, launch after launch, under CUDA-graph replay, at
M = 1, 3 and with fp32 outputs; the chain's flags and launch counts advance
once per launch and no wait gives up.
"""
from __future__ import annotations

import pytest
import torch

from drinkme_b200 import codec, radix_ops, shard, swap

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)

# (rows, cols): each link's cols equal the previous link's rows, so link k
# reads link k-1's gathered output; the last one reads a fixed input.
# Ragged rows (1000), a tensor with resident activations (NB <= 16) and one
# staged per unit (NB = 20).
SHAPES = ((2048, 1024), (1024, 2048), (4096, 1024), (1000, 4096), (512, 20480))


def _tensors():
    g = torch.Generator().manual_seed(7)
    rts = []
    for R, C in SHAPES:
        W = (torch.randn(R, C, generator=g) * 0.02).to(torch.bfloat16)
        rts.append(swap.to_device_radix(codec.pack_weight_radix(W, "sip"), DEV))
    return rts


@pytest.mark.parametrize("M,dtype", [(1, torch.bfloat16), (3, torch.bfloat16), (2, torch.float32)])
def test_chain_equals_per_linear_calls(M, dtype):
    rts = _tensors()
    g = torch.Generator().manual_seed(8)
    x0 = torch.randn(M, SHAPES[0][1], generator=g).to(torch.bfloat16).to(DEV)
    xl = torch.randn(M, SHAPES[-1][1], generator=g).to(torch.bfloat16).to(DEV)
    plan = shard.PeerGather([R for R, _ in SHAPES], M, dtype, 0, 1, DEV)
    chain = None
    try:
        links = []
        for k, rt in enumerate(rts):
            if k == 0:
                x, wait = x0, len(rts) - 1  # the previous launch's last link
            elif k == len(rts) - 1:
                x, wait = xl, k - 1
            else:
                # an earlier link's output as this one's input (bf16 chains only)
                x = plan.output(k - 1)[:, :SHAPES[k][1]] if dtype == torch.bfloat16 else \
                    torch.randn(M, SHAPES[k][1], generator=g).to(torch.bfloat16).to(DEV)
                wait = k - 1
            links.append((rt, x, k, wait, None))
        chain = plan.chain(links)
        # the per-linear calls on the same activations, link by link
        want = []
        for k, (rt, x, _, _, _) in enumerate(links):
            xin = want[k - 1][:, :SHAPES[k][1]] if (0 < k < len(rts) - 1 and dtype == torch.bfloat16) else x
            want.append(radix_ops.gemv_mc_fused(rt, xin.contiguous(), None, dtype))
        for launch in range(1, 4):
            chain.run()
            torch.cuda.synchronize()
            for k in range(len(rts)):
                assert torch.equal(plan.output(k)[:, :SHAPES[k][0]], want[k]), (launch, k)
                assert int(plan.launch_count(k)) == launch
        # captured in a CUDA graph and replayed
        s = torch.cuda.Stream(DEV)
        s.wait_stream(torch.cuda.current_stream(DEV))
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            chain.run()
        for _ in range(2):
            graph.replay()
        torch.cuda.synchronize()
        for k in range(len(rts)):
            assert torch.equal(plan.output(k)[:, :SHAPES[k][0]], want[k]), ("graph", k)
            assert int(plan.launch_count(k)) == 5
        del graph
        assert int(plan.abort_word()) == 0
        assert all(rt["rx_handle"].device_error() == 0 for rt in rts)
    finally:
        if chain is not None:
            chain.close()
        plan.close()


def test_chain_refuses_bad_links():
    rts = _tensors()[:2]
    x = torch.zeros(1, SHAPES[0][1], dtype=torch.bfloat16, device=DEV)
    plan = shard.PeerGather([R for R, _ in SHAPES[:2]], 1, torch.bfloat16, 0, 1, DEV)
    try:
        with pytest.raises(ValueError, match="wait index"):
            plan.chain([(rts[0], x, 0, 5, None)])
        with pytest.raises(ValueError, match="16-byte aligned"):
            buf = torch.zeros(1, SHAPES[0][1] + 1, dtype=torch.bfloat16, device=DEV)
            plan.chain([(rts[0], buf[:, 1:], 0, None, None)])
    finally:
        plan.close()


def test_chain_wait_that_never_completes_returns_with_an_error():
    """A link whose predecessor's CTA count never reaches this run's target
    (reset by hand after the first run) gives up after its poll bound,
    records kErrWaitPeer (4) in its tensor's error word and sets the abort
    word; the launch still ends and the GPU stays usable (a plain GEMV
    afterwards equals the first run's output)."""
    from drinkme_b200.tensor import device_view

    rts = _tensors()[:2]
    x = torch.randn(1, SHAPES[0][1], generator=torch.Generator().manual_seed(9)).to(torch.bfloat16).to(DEV)
    plan = shard.PeerGather([R for R, _ in SHAPES[:2]], 1, torch.bfloat16, 0, 1, DEV)
    chain = None
    try:
        chain = plan.chain([(rts[0], x, 0, None, None), (rts[1], plan.output(0)[:, :SHAPES[1][1]], 1, 0, None)],
                           wait_polls=1 << 12)
        chain.run()
        torch.cuda.synchronize()
        want = plan.output(1)[:, :SHAPES[1][0]].clone()
        assert rts[1]["rx_handle"].device_error() == 0 and int(plan.abort_word()) == 0
        # link 0's CTA count (the word after its launch count) back to zero:
        # the next run's link 1 waits for a count it never sees
        device_view(plan.base + plan.cnt_off + 4, (1,), torch.int32, DEV).fill_(0)
        chain.run()
        torch.cuda.synchronize()
        assert rts[1]["rx_handle"].device_error() == 4  # kErrWaitPeer
        assert int(plan.abort_word()) != 0
        y = radix_ops.gemv_mc_fused(rts[1], plan.output(0)[:, :SHAPES[1][1]].contiguous(), None, torch.bfloat16)
        assert torch.equal(y, want)
    finally:
        if chain is not None:
            chain.close()
        plan.close()
