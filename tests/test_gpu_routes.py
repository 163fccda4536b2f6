"""The module's row routes on B200 (swap.CompressedLinear; reference
swap.py:302-392, serving/mtp.py:228-240): an MTP verify batch of up to
fused_m_max() rows, and the row loop between MC_MAX and the measured dense
threshold (through the multi-column kernel in chunks of MC_MAX rows), give
every row bitwise the serial one-row step's answer; the dense arm above the
threshold stays within the float64 bound (bf16 activations; fp32 ones meet
the reference's F.linear dtype rule there)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from drinkme_b200 import codec, swap
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_verify_batch_and_row_loop_are_the_serial_steps(dtype):
    g = torch.Generator().manual_seed(8)
    W = (torch.randn(1000, 4096, generator=g) * 0.02).to(torch.bfloat16)
    bias = (torch.randn(1000, generator=g) * 0.1).to(torch.bfloat16).to(DEV)
    m = swap.make_module(codec.pack_weight_radix(W, "sip"), bias, DEV)
    x = torch.randn(24, 4096, generator=g).to(dtype).to(DEV)
    swap._DENSE_MIN = None
    serial = torch.cat([m(x[i:i + 1]) for i in range(24)])
    k = swap.fused_m_max()
    assert k == 8 and m._route(x[:k]) == "mc"
    for M in (2, 5, k):  # MTP verify widths (drafts + 1)
        assert torch.equal(m(x[:M]), serial[:M]), M
    for M in (9, 12, 16):
        assert m._route(x[:M]) == "loop"
        assert torch.equal(m(x[:M]), serial[:M]), M
    assert m._route(x[:17]) == "dense"
    if dtype == torch.float32:
        # the dense arm is F.linear over the bf16 weight, as the reference's
        # (swap.py:376): fp32 activations meet a bf16 weight and torch refuses
        with pytest.raises(RuntimeError):
            m(x[:17])
        return
    y = m(x[:17]).float().cpu().numpy()
    y64, bound = oracle.gemv_bound(x[:17].float().cpu().numpy(), codec.bits_of(W))
    y64 = y64 + bias.float().cpu().numpy()
    # the dense arm rounds its GEMM output once to x's dtype (bf16: 2^-8 relative)
    slack = np.abs(y64) * (2.0 ** -8 if dtype == torch.bfloat16 else 2.0 ** -20)
    assert np.all(np.abs(y - y64) <= bound + slack + 1e-6)
