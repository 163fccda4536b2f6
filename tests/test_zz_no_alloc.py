"""dm_gemv_noalloc — the GEMV entry point for callers that cannot allocate
device memory when they call it (a serving engine whose HBM already belongs
to its own pool, a decode loop that must not risk cudaMalloc's device
synchronisation). Its scratch is one static array in the library's device
memory instead of the tensor's own buffers; everything else is dm_gemv.

Called through the C ABI, twice in a row (the array keeps the first call's
contents), it must give dm_gemv's outputs — bitwise, as both run the same
kernel over the same split — and stay within the float64 bound every GEMV test
here uses. Named to be collected last: if it fails, a run that stops at the
first failure has already run every other test.
"""
from __future__ import annotations

import ctypes as ct

import numpy as np
import pytest
import torch

from drinkme_b200 import _lib, codec, swap
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
_DT = {torch.bfloat16: _lib.DM_BF16, torch.float32: _lib.DM_F32}


def _call(fn, rt, x, bias, out):
    h = rt["rx_handle"]
    stream = ct.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)
    _lib.call(fn, h.ptr, ct.c_void_p(x.data_ptr()), _DT[x.dtype], x.shape[0],
              ct.c_void_p(bias.data_ptr() if bias is not None else 0), ct.c_void_p(out.data_ptr()),
              _DT[out.dtype], stream)
    return out


def _tensor(R, C, profile, seed):
    g = torch.Generator().manual_seed(seed)
    W = (torch.randn(R, C, generator=g) * 0.02).to(torch.bfloat16)
    p = codec.pack_weight_radix(W, profile)
    return swap.to_device_radix(p, DEV), codec.bits_of(W)


@pytest.mark.parametrize("R,C,profile", [(4096, 12288, "sip"), (1000, 4096, "sip"), (300, 4096, "gulp")])
@pytest.mark.parametrize("M,xdt,odt", [(1, torch.bfloat16, torch.bfloat16), (3, torch.bfloat16, torch.float32),
                                       (2, torch.float32, torch.float32)])
def test_noalloc_matches_dm_gemv_on_two_calls_in_a_row(R, C, profile, M, xdt, odt):
    rt, bits = _tensor(R, C, profile, seed=R + C)
    g = torch.Generator().manual_seed(7)
    x = torch.randn(M, C, generator=g).to(xdt).to(DEV)
    bias = (torch.randn(R, generator=g) * 0.1).to(torch.bfloat16).to(DEV)
    ref = _call("dm_gemv", rt, x, bias, torch.empty(M, R, dtype=odt, device=DEV))
    for _ in range(2):
        got = _call("dm_gemv_noalloc", rt, x, bias, torch.full((M, R), float("nan"), dtype=odt, device=DEV))
        torch.cuda.synchronize()
        assert torch.equal(got, ref)
    nb = _call("dm_gemv_noalloc", rt, x, None, torch.empty(M, R, dtype=torch.float32, device=DEV))
    y64, bound = oracle.gemv_bound(x.float().cpu().numpy(), bits)
    assert np.all(np.abs(nb.cpu().numpy() - y64) <= bound)
    assert rt["rx_handle"].device_error() == 0


def test_noalloc_refuses_sizes_beyond_its_static_scratch():
    rt, _ = _tensor(16, 33 * 1024, "sip", seed=3)
    x = torch.randn(1, 33 * 1024, device=DEV)
    with pytest.raises(ValueError, match="exceed the static scratch"):
        _call("dm_gemv_noalloc", rt, x, None, torch.empty(1, 16, dtype=torch.float32, device=DEV))
    xb = x.to(torch.bfloat16)  # aligned bf16 activations need no staging: served
    y = _call("dm_gemv_noalloc", rt, xb, None, torch.empty(1, 16, dtype=torch.float32, device=DEV))
    assert torch.equal(y, _call("dm_gemv", rt, xb, None, torch.empty(1, 16, dtype=torch.float32, device=DEV)))


def test_noalloc_refuses_m_outside_one_to_eight():
    rt, _ = _tensor(64, 4096, "sip", seed=4)
    with pytest.raises(ValueError, match="outside 1"):
        _call("dm_gemv_noalloc", rt, torch.zeros(9, 4096, dtype=torch.bfloat16, device=DEV), None,
              torch.empty(9, 64, dtype=torch.bfloat16, device=DEV))


@pytest.mark.parametrize("xdt", [torch.bfloat16, torch.float32])
def test_noalloc_misaligned_activations_match_dm_gemv(xdt):
    """Activations one element past a 16-byte boundary are staged into the
    static array (copied, or split for fp32) and give dm_gemv's bits."""
    rt, bits = _tensor(4096, 12288, "sip", seed=31)
    g = torch.Generator().manual_seed(8)
    for M in (1, 3, 8):
        buf = torch.empty(M * 12288 + 1, dtype=xdt, device=DEV)
        buf[1:] = torch.randn(M * 12288, generator=g).to(xdt).to(DEV)
        x = buf[1:].view(M, 12288)
        assert x.data_ptr() % 16 != 0
        ref = _call("dm_gemv", rt, x, None, torch.empty(M, 4096, dtype=torch.float32, device=DEV))
        for _ in range(2):
            got = _call("dm_gemv_noalloc", rt, x, None, torch.full((M, 4096), float("nan"), device=DEV))
            assert torch.equal(got, ref)
        y64, bound = oracle.gemv_bound(x.float().cpu().numpy(), bits)
        assert np.all(np.abs(ref.cpu().numpy() - y64) <= bound)
    assert rt["rx_handle"].device_error() == 0


def test_noalloc_calls_allocate_no_device_memory():
    """After a first call (which looks the array's address up), further calls
    of every kind leave the device's free memory unchanged."""
    rt, _ = _tensor(4096, 12288, "sip", seed=32)
    g = torch.Generator().manual_seed(9)
    xs = [torch.randn(2, 12288, generator=g).to(torch.bfloat16).to(DEV),
          torch.randn(3, 12288, generator=g).to(DEV)]
    buf = torch.empty(2 * 12288 + 1, dtype=torch.bfloat16, device=DEV)
    xs.append(buf[1:].view(2, 12288))
    outs = [torch.empty(x.shape[0], 4096, dtype=torch.float32, device=DEV) for x in xs]
    for x, o in zip(xs, outs):
        _call("dm_gemv_noalloc", rt, x, None, o)
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        for x, o in zip(xs, outs):
            _call("dm_gemv_noalloc", rt, x, None, o)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
