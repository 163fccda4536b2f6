"""GPU: the entry points at any activation alignment, and the ordering of
back-to-back launches on one stream.

The reference's arms accept any contiguous x (radix_ops.py:379-398), which a
view at an odd element offset is. The sip kernel stages activations with bulk
copies that need 16-byte aligned sources, and its layout holds each block's
tier-0 codes as code planes that only the sip kernels read, so such x is
copied (bf16) or split (fp32) to an aligned buffer first: the result must be
the aligned call's bits, and within the float64 bound of the oracle.

The sip kernels start early under programmatic dependent launch; the decode
mode, which reads no activations, must still wait for the kernel before it
before storing into memory that kernel may use.
"""
from __future__ import annotations

import ctypes as ct

import numpy as np
import pytest
import torch

from drinkme_b200 import _lib, codec, radix_ops, swap
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _tensor(R, C, seed, profile="sip"):
    g = torch.Generator().manual_seed(seed)
    W = (torch.randn(R, C, generator=g) * 0.02).to(torch.bfloat16)
    return swap.to_device_radix(codec.pack_weight_radix(W, profile), DEV), codec.bits_of(W)


def _misaligned(M, C, dtype, seed):
    """[M, C] activations one element past a 16-byte boundary."""
    g = torch.Generator().manual_seed(seed)
    buf = torch.empty(M * C + 1, dtype=dtype, device=DEV)
    buf[1:] = torch.randn(M * C, generator=g).to(dtype).to(DEV)
    x = buf[1:].view(M, C)
    assert x.data_ptr() % 16 != 0
    return x


@pytest.fixture(scope="module")
def tensors():
    return {"config1": _tensor(4096, 12288, seed=11), "ragged40": _tensor(40, 4096, seed=12)}


@pytest.mark.parametrize("name", ["config1", "ragged40"])
@pytest.mark.parametrize("M", [1, 3, 8])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_misaligned_activations_match_aligned_and_oracle(tensors, name, M, dtype):
    rt, bits = tensors[name]
    assert radix_ops.decoder_of(rt) == radix_ops.DECODER_SIP_MMA
    x = _misaligned(M, bits.shape[1], dtype, seed=M)
    y = radix_ops.gemv_mc(rt, x)
    assert torch.equal(y, radix_ops.gemv_mc(rt, x.clone()))
    y64, bound = oracle.gemv_bound(x.float().cpu().numpy(), bits)
    assert np.all(np.abs(y.cpu().numpy().astype(np.float64) - y64) <= bound)
    # the fused epilogue too: bias in fp32, one rounding
    bias = torch.randn(bits.shape[0], generator=torch.Generator().manual_seed(5)).to(torch.bfloat16).to(DEV)
    yb = radix_ops.gemv_mc_fused(rt, x, bias, torch.bfloat16)
    assert torch.equal(yb, (y + bias.float()).to(torch.bfloat16))
    assert rt["rx_handle"].device_error() == 0


def test_generic_kernel_never_reads_a_code_plane_layout(tensors):
    """The general kernel refuses a sip fast-path handle (C++ check in its
    launcher); only packs the sip kernels cannot serve reach it."""
    rt, _ = tensors["ragged40"]
    assert rt["rx_handle"].info.fast_path == 1
    rg, bits = _tensor(40, 1000, seed=13)  # ragged block: the general kernel
    assert radix_ops.decoder_of(rg) == radix_ops.DECODER_GENERIC
    x = _misaligned(2, 1000, torch.bfloat16, seed=4)
    y64, bound = oracle.gemv_bound(x.float().cpu().numpy(), bits)
    assert np.all(np.abs(radix_ops.gemv_mc(rg, x).cpu().numpy() - y64) <= bound)


def test_activations_off_their_element_size_are_refused(tensors):
    rt, _ = tensors["ragged40"]
    buf = torch.zeros(4 * 4096 + 4, dtype=torch.uint8, device=DEV)
    out = torch.empty(1, 40, dtype=torch.float32, device=DEV)
    for dt, off in ((_lib.DM_BF16, 1), (_lib.DM_F32, 2)):
        with pytest.raises(ValueError, match="element size"):
            _lib.call("dm_gemv", rt["rx_handle"].ptr, ct.c_void_p(buf.data_ptr() + off), dt, 1, ct.c_void_p(0),
                      ct.c_void_p(out.data_ptr()), _lib.DM_F32,
                      ct.c_void_p(torch.cuda.current_stream(DEV).cuda_stream))


def test_raw_gemv_serves_misaligned_inputs():
    """dm_gemv_raw takes its scalar loop for a weight or activations off a
    16-byte boundary instead of refusing them."""
    g = torch.Generator().manual_seed(21)
    wbuf = (torch.randn(64 * 1024 + 1, generator=g) * 0.02).to(torch.bfloat16).to(DEV)
    w = wbuf[1:].view(64, 1024)
    x = _misaligned(3, 1024, torch.bfloat16, seed=22)
    y = radix_ops.gemv_raw(w, x, None, torch.float32)
    assert torch.equal(y, radix_ops.gemv_raw(w, x, None, torch.float32))  # deterministic
    bits = w.cpu().view(torch.int16).numpy().view(np.uint16)
    y64, bound = oracle.gemv_bound(x.float().cpu().numpy(), bits)
    assert np.all(np.abs(y.cpu().numpy() - y64) <= bound)


def test_back_to_back_decodes_into_one_buffer(tensors):
    """Two decode launches into the same output, then a GEMV over other
    memory and a decode into the GEMV's output block once torch frees it:
    every decode must land whole (the decode mode waits for the kernel
    before it before storing)."""
    rt, bits = tensors["config1"]
    ref = torch.from_numpy(bits.view(np.int16)).to(DEV)
    out = torch.empty_like(ref)
    h = rt["rx_handle"]
    stream = ct.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)
    for _ in range(3):
        out.fill_(0)
        _lib.call("dm_decode", h.ptr, ct.c_void_p(out.data_ptr()), stream)
        _lib.call("dm_decode", h.ptr, ct.c_void_p(out.data_ptr()), stream)
        assert torch.equal(out, ref)
    # a GEMV whose output block the caching allocator hands to the decode next
    x = torch.randn(8, 12288, generator=torch.Generator().manual_seed(9)).to(torch.bfloat16).to(DEV)
    for _ in range(3):
        y = torch.empty(4096 * 12288 // 2, dtype=torch.float32, device=DEV)  # the size of the decode output
        radix_ops.gemv_into(rt, x, None, y[: 8 * 4096].view(8, 4096))
        del y  # usually the block decode_bits gets next, on the same stream
        assert torch.equal(radix_ops.decode_bits(rt).view(torch.int16), ref)
    assert h.device_error() == 0
