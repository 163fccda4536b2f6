"""The prefill kernel (dm_prefill, radix_ops.prefill): sip weights decoded
into shared memory and contracted on the tensor cores (tcgen05.mma, fp32
accumulate in tensor memory).

Gates: fp32 outputs within |y - y64| <= 2e-6 * |x|.|W| + 1e-7 of float64
(the reference's bound, bench/radix_gemv_bitpin.py:182) and within 1e-3 max
relative error of F.linear over the decoded weight; the bias added in fp32
before one rounding; every activation-row count from 1 through several
512-row passes, ragged weight tiles, the config-5 shapes; repeated calls
bitwise equal.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from drinkme_b200 import codec, radix_ops, swap
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _case(R, C, M, seed):
    g = torch.Generator().manual_seed(seed)
    W = (torch.randn(R, C, generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn(M, C, generator=g).to(torch.bfloat16)
    rt = swap.to_device_radix(codec.pack_weight_radix(W, "sip"), DEV)
    return W, x, rt


def _check(y, x, W):
    y = y.float().cpu().numpy()
    y64, bound = oracle.gemv_bound(x.float().numpy(), codec.bits_of(W))
    err = np.abs(y.astype(np.float64) - y64)
    assert np.all(err <= bound), float((err / bound).max())
    assert np.abs(y - y64).max() / max(np.abs(y64).max(), 1e-30) <= 1e-3


@pytest.mark.parametrize("R,C,M", [(128, 1024, 128), (256, 4096, 9), (300, 4096, 200), (1024, 2048, 512),
                                   (160, 3072, 600), (64, 8192, 1), (1000, 1024, 33)])
def test_prefill_within_float64_bound(R, C, M):
    W, x, rt = _case(R, C, M, seed=R + C + M)
    y = radix_ops.prefill(rt, x.to(DEV), None, torch.float32)
    _check(y, x, W)
    assert torch.equal(y, radix_ops.prefill(rt, x.to(DEV), None, torch.float32))
    assert rt["rx_handle"].device_error() == 0


def test_prefill_bias_rounds_once_and_matches_dense_arm():
    W, x, rt = _case(384, 4096, 130, seed=5)
    xd = x.to(DEV)
    bias = (torch.randn(384, generator=torch.Generator().manual_seed(6)) * 0.5).to(torch.bfloat16).to(DEV)
    y32 = radix_ops.prefill(rt, xd, None, torch.float32)
    yb = radix_ops.prefill(rt, xd, bias, torch.bfloat16)
    assert torch.equal(yb, (y32 + bias.float()).to(torch.bfloat16))
    dense = torch.nn.functional.linear(xd.float(), radix_ops.decode_weight(rt).float())
    assert (y32 - dense).abs().max() / dense.abs().max() <= 1e-3


def test_prefill_config5_shapes():
    """x [512, 4096] against gate 12288x4096; down 4096x12288."""
    for R, C, seed in ((12288, 4096, 1), (4096, 12288, 2)):
        W, x, rt = _case(R, C, 512, seed)
        y = radix_ops.prefill(rt, x.to(DEV), None, torch.float32)
        ref = torch.nn.functional.linear(x.to(DEV).float(), W.to(DEV).float())
        assert (y - ref).abs().max() / ref.abs().max() <= 1e-3
        _check(y[:64], x[:64], W)


def test_prefill_escape_heavy_rows_and_fused_parts():
    """Exponents spread far past the sip palette: most weights escape, so
    ranks run past the 64 terminal bytes staged per row (the rest come from
    HBM); a fused q|k|v-like tensor (three parts, three palettes) and a row
    shard; activations off a 16-byte boundary."""
    g = torch.Generator().manual_seed(71)
    base = torch.randn(200, 2048, generator=g) * 0.02
    wild = torch.rand(200, 2048, generator=g) < 0.15  # about 150 escapes per block
    scale = torch.pow(2.0, torch.randint(-60, 60, (200, 2048), generator=g).float())
    W = torch.where(wild, base * scale, base).to(torch.bfloat16)
    p = codec.pack_weight_radix(W, "sip")
    assert p["codec"] == "radix"
    rt = swap.to_device_radix(p, DEV)
    x = torch.randn(70, 2048, generator=g).to(torch.bfloat16)
    buf = torch.empty(70 * 2048 + 1, dtype=torch.bfloat16, device=DEV)
    buf[1:] = x.reshape(-1).to(DEV)
    y = radix_ops.prefill(rt, buf[1:].view(70, 2048), None, torch.float32)
    _check(y, x, W)
    Ws = [(torch.randn(r, 4096, generator=g) * s).to(torch.bfloat16) for r, s in ((256, 0.02), (64, 0.05), (64, 1.0))]
    packs = [codec.pack_weight_radix(w, "sip") for w in Ws]
    fused = swap.to_device_radix_fused(packs, DEV)
    xf = torch.randn(40, 4096, generator=g).to(torch.bfloat16)
    yf = radix_ops.prefill(fused, xf.to(DEV), None, torch.float32)
    _check(yf, xf, torch.cat(Ws))
    shard = swap.to_device_radix(packs[0], DEV, 64, 192)
    _check(radix_ops.prefill(shard, xf.to(DEV), None, torch.float32), xf, Ws[0][64:192])
    assert rt["rx_handle"].device_error() == 0 and fused["rx_handle"].device_error() == 0


@pytest.mark.parametrize("M", [9, 96, 257, 1100])
def test_prefill_token_tiles_and_stream_k_pieces(M):
    """Activation-row counts that leave partial token tiles, several token
    tiles and (on the 8B down shape) tiles shared by several CTAs."""
    W, x, rt = _case(4096, 12288, M, seed=M)
    y = radix_ops.prefill(rt, x.to(DEV), None, torch.float32)
    ref = torch.nn.functional.linear(x.to(DEV).float(), W.to(DEV).float())
    assert (y - ref).abs().max() / ref.abs().max() <= 1e-3
    _check(y[: min(M, 24)], x[: min(M, 24)], W)
    assert torch.equal(y, radix_ops.prefill(rt, x.to(DEV), None, torch.float32))
    assert rt["rx_handle"].device_error() == 0
