"""Fused tensors on the GPU (dm_tensor_create_multi): the rows of several sip
packs reading the same activations — q, k, v or gate, up — served by one
launch. Each part keeps its own palette (its exponent tables travel in the
unit headers), so the gates are those of a single tensor, per part:

  * decode bit-exact: the stacked bits of every part;
  * GEMV within |y - y64| <= 2e-6 * |x|.|W| + 1e-7 of float64 over the
    stacked weight, for M = 1..8, bf16 and fp32 activations;
  * the fused bias rounds once; row m of an M-row call bitwise the M=1 call.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from drinkme_b200 import codec, radix_ops, swap
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _weights(shapes, C, seed):
    """Parts with different scales, so their palettes (exponent ranks) differ."""
    g = torch.Generator().manual_seed(seed)
    return [(torch.randn(r, C, generator=g) * s).to(torch.bfloat16) for r, s in zip(shapes, (0.02, 0.3, 4.0, 1e-3))]


def _fused(Ws, ranges=None):
    packs = [codec.pack_weight_radix(W, "sip") for W in Ws]
    assert len({bytes(p["rx_palette"][:7]) for p in packs}) > 1, "palettes should differ"
    return swap.to_device_radix_fused(packs, DEV, ranges), packs


def _within_bound(y, x, bits):
    y64, bound = oracle.gemv_bound(x.float().cpu().numpy(), bits)
    err = np.abs(y.astype(np.float64) - y64)
    return bool(np.all(err <= bound)), float((err / bound).max())


@pytest.mark.parametrize("shapes,C", [((256, 64, 64), 4096), ((512, 512), 8192), ((32, 48, 16, 100), 4096),
                                      ((16, 13), 2048)])
def test_fused_decode_and_gemv(shapes, C):
    Ws = _weights(shapes, C, seed=sum(shapes) + C)
    rt, _ = _fused(Ws)
    assert radix_ops.decoder_of(rt) == radix_ops.DECODER_SIP_MMA
    assert rt["R"] == sum(shapes) and rt["fused_rows"] == tuple(shapes)
    bits = np.concatenate([codec.bits_of(W) for W in Ws])
    assert np.array_equal(radix_ops.decode_bits(rt).cpu().numpy().view(np.uint16), bits)
    g = torch.Generator().manual_seed(11)
    x = torch.randn(8, C, generator=g)
    for dt in (torch.bfloat16, torch.float32):
        xd = x.to(dt).to(DEV)
        y1 = radix_ops.gemv_mc(rt, xd[:1])
        for M in (1, 3, 8):
            y = radix_ops.gemv_mc(rt, xd[:M])
            ok, worst = _within_bound(y.cpu().numpy(), xd[:M], bits)
            assert ok, (shapes, dt, M, worst)
            assert torch.equal(y[0], y1[0])
    assert rt["rx_handle"].device_error() == 0


def test_fused_parts_split_and_bias_rounds_once():
    Ws = _weights((128, 32, 32), 4096, seed=3)
    rt, _ = _fused(Ws)
    g = torch.Generator().manual_seed(4)
    x = torch.randn(2, 4096, generator=g).to(torch.bfloat16).to(DEV)
    bias = (torch.randn(192, generator=g)).to(torch.bfloat16).to(DEV)
    y32 = radix_ops.gemv_mc(rt, x)
    yb = radix_ops.gemv_mc_fused(rt, x, bias, torch.bfloat16)
    assert torch.equal(yb, (y32 + bias.float()).to(torch.bfloat16))
    q, k, v = swap.split_fused(rt, y32)
    assert q.shape == (2, 128) and k.shape == (2, 32) and v.shape == (2, 32)
    for part, W in zip((q, k, v), Ws):
        ok, worst = _within_bound(part.cpu().numpy(), x, codec.bits_of(W))
        assert ok, worst


def test_fused_row_shards():
    """A rank's shard of each projection, fused: rows [r0, r1) of every part."""
    Ws = _weights((256, 64, 64), 4096, seed=9)
    packs = [codec.pack_weight_radix(W, "sip") for W in Ws]
    x = torch.randn(1, 4096, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16).to(DEV)
    for ranges in (((0, 128), (0, 32), (0, 32)), ((128, 256), (32, 64), (32, 64))):
        rt = swap.to_device_radix_fused(packs, DEV, ranges)
        bits = np.concatenate([codec.bits_of(W)[a:b] for W, (a, b) in zip(Ws, ranges)])
        assert np.array_equal(radix_ops.decode_bits(rt).cpu().numpy().view(np.uint16), bits)
        ok, worst = _within_bound(radix_ops.gemv_mc(rt, x).cpu().numpy(), x, bits)
        assert ok, worst


def test_fused_tensor_serves_misaligned_activations():
    """Activations off a 16-byte boundary (a view at an odd element offset)
    are staged to an aligned copy: the same bits as the aligned call."""
    Ws = _weights((16, 16), 1024, seed=1)
    rt, _ = _fused(Ws)
    buf = torch.randn(1025, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16).to(DEV)
    x = buf[1:].reshape(1, 1024)
    assert x.data_ptr() % 16 != 0
    assert torch.equal(radix_ops.gemv_mc(rt, x), radix_ops.gemv_mc(rt, x.clone()))


def test_fused_sip_and_reencoded_gulp_parts():
    """A gulp part with whole 1024-weight blocks is re-encoded as sip by the
    loader and fuses with sip parts; every part's bits stay exact."""
    Ws = _weights((128, 64), 4096, seed=17)
    packs = [codec.pack_weight_radix(Ws[0], "sip"), codec.pack_weight_radix(Ws[1], "gulp")]
    rt = swap.to_device_radix_fused(packs, DEV)
    bits = np.concatenate([codec.bits_of(W) for W in Ws])
    assert np.array_equal(radix_ops.decode_bits(rt).cpu().numpy().view(np.uint16), bits)
    x = torch.randn(4, 4096, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16).to(DEV)
    ok, worst = _within_bound(radix_ops.gemv_mc(rt, x).cpu().numpy(), x, bits)
    assert ok, worst
