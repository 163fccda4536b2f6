"""GPU: the launch schedule reaches the kernel. The b200 table row (or the
DRINKME_RADIX_SCHEDULE override, the reference's configuration surface:
radix_schedule.py:372-417) sets a tensor's launch knobs at load; dm_gemv_plan
reports the launch they make. Slots and residency change the staging only:
the same result bits. The split changes which CTA sums which units: results
stay within the float64 bound. Decoded weights are the same bits under every
launch."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from drinkme_b200 import codec, radix_ops, swap
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(scope="module")
def packed():
    g = torch.Generator().manual_seed(51)
    W = (torch.randn(4096, 12288, generator=g) * 0.02).to(torch.bfloat16)
    return codec.pack_weight_radix(W, "sip"), codec.bits_of(W)


def _x(M, C=12288):
    return torch.randn(M, C, generator=torch.Generator().manual_seed(M)).to(torch.bfloat16).to(DEV)


def test_override_changes_the_launch_not_the_bits(packed, monkeypatch):
    p, bits = packed
    base = swap.to_device_radix(p, DEV)
    h = base["rx_handle"]
    plan0 = h.plan(1)
    assert plan0["slots"] == 6 and plan0["resident"] == 1 and plan0["grid"] == 148
    xs = {M: _x(M) for M in (1, 4)}
    ref = {M: radix_ops.gemv_mc(base, x) for M, x in xs.items()}
    dec = radix_ops.decode_bits(base).cpu().numpy()
    for spec, want in (("slots=3", dict(slots=3)), ("resident=0", dict(resident=0)),
                       ("slots=2,resident=0", dict(slots=2, resident=0))):
        monkeypatch.setenv("DRINKME_RADIX_SCHEDULE", spec)
        rt = swap.to_device_radix(p, DEV)
        assert rt["rx_launch"]["source"] == "env"
        plan = rt["rx_handle"].plan(1)
        for k, v in want.items():
            assert plan[k] == v, (spec, plan)
        for M, x in xs.items():
            assert torch.equal(radix_ops.gemv_mc(rt, x), ref[M]), (spec, M)
        assert np.array_equal(radix_ops.decode_bits(rt).cpu().numpy(), dec)
    monkeypatch.setenv("DRINKME_RADIX_SCHEDULE", "split=tiles")
    rt = swap.to_device_radix(p, DEV)
    assert rt["rx_handle"].plan(1)["split"] == 2 and plan0["split"] == 1
    for M, x in xs.items():
        y64, bound = oracle.gemv_bound(x.float().cpu().numpy(), bits)
        assert np.all(np.abs(radix_ops.gemv_mc(rt, x).cpu().numpy() - y64) <= bound)
    assert np.array_equal(radix_ops.decode_bits(rt).cpu().numpy(), dec)
    monkeypatch.setenv("DRINKME_RADIX_SCHEDULE", "spike")
    rt = swap.to_device_radix(p, DEV)
    plan = rt["rx_handle"].plan(1)
    assert plan["split"] == 2 and plan["slots"] == 2 and plan["resident"] == 0
    y64, bound = oracle.gemv_bound(xs[1].float().cpu().numpy(), bits)
    assert np.all(np.abs(radix_ops.gemv_mc(rt, xs[1]).cpu().numpy() - y64) <= bound)
    assert h.device_error() == 0 and rt["rx_handle"].device_error() == 0


def test_set_launch_refuses_out_of_range_knobs(packed):
    p, _ = packed
    h = swap.to_device_radix(p, DEV)["rx_handle"]
    for kw in (dict(slots=7), dict(split=3), dict(skew=65), dict(resident=17)):
        with pytest.raises(ValueError):
            h.set_launch(**kw)
    h.set_launch(skew=0)
    assert h.plan(1)["skew_step"] == 0
    h.set_launch(skew=8)
    assert h.plan(1)["skew_step"] > 0
