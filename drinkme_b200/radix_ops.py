"""The radix operator arms over a to_device_radix runtime dict — the drop-in
for the reference's ``drinkme.codec.radix_ops`` (src/drinkme/codec/
radix_ops.py), same function names, arguments and errors, served by the
sm_100a kernels of libdrinkme_b200.so through its C ABI:

  gemv_fused(p, x, bias, out_dtype)   radix_ops.py:351-370  the M=1 arm
  gemv(p, x)                          radix_ops.py:373-376  fp32 [R], no bias
  gemv_mc(p, x)                       radix_ops.py:379-398  1 <= M <= MC_MAX
  gemv_narrow(w, x, bias, block, nw)  radix_ops.py:401-415  raw bf16 weight
  decode_bits(p) / decode_weight(p)   radix_ops.py:418-432
  prepare_schedule(...)               radix_ops.py:341-348
  read_bytes(p)                       radix_ops.py:435-441

Every arm runs on the tensor's CUDA device on torch's current stream; there
is no CPU route here and no fallback — the library must be built.
"""
from __future__ import annotations

import ctypes as ct

import torch

from . import _lib
from .ops import MC_MAX

DECODER_SIP_MMA = "sip-mma-sm100a"   # the fused decode + MMA kernel (sip, 1024-weight blocks)
DECODER_GENERIC = "generic-sm100a"   # any widths / block size / ragged rows

_DT = {torch.bfloat16: _lib.DM_BF16, torch.float32: _lib.DM_F32}


def _stream(dev: torch.device) -> ct.c_void_p:
    return ct.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _handle(p: dict):
    h = p.get("rx_handle")
    if h is None:
        raise ValueError("radix_ops: not a drinkme_b200 runtime dict (to_device_radix builds one)")
    return h


def decoder_of(p: dict) -> str:
    """Which kernel serves this tensor's GEMV / MC arm."""
    return DECODER_SIP_MMA if _handle(p).info.fast_path else DECODER_GENERIC


def _check_x(x: torch.Tensor, C: int, dev: torch.device) -> torch.Tensor:
    if x.device != dev:
        raise ValueError(f"radix_ops: activations on {x.device}, tensor on {dev}")
    if x.dtype not in _DT:
        raise TypeError(f"radix_ops: activations must be bf16 or fp32, not {x.dtype}")
    if x.shape[-1] != C:
        raise ValueError(f"radix_ops: activations have {x.shape[-1]} columns, the tensor {C}")
    return x.contiguous()


def _run(p: dict, x: torch.Tensor, bias, out_dtype, out: torch.Tensor | None = None) -> torch.Tensor:
    h = _handle(p)
    dev = h.torch_device
    x = _check_x(x, h.info.C, dev)
    M = x.shape[0]
    if not 1 <= M <= MC_MAX:
        raise ValueError(f"radix gemv_mc: M={M} outside 1..{MC_MAX}")
    if out_dtype not in _DT:
        raise TypeError(f"radix_ops: output dtype must be bf16 or fp32, not {out_dtype}")
    rows = h.info.rows
    if out is None:
        out = torch.empty((M, rows), dtype=out_dtype, device=dev)
    elif out.dtype != out_dtype or out.numel() != M * rows or not out.is_contiguous() or out.device != dev:
        raise ValueError("radix_ops: `out` must be a contiguous [M, rows] tensor of the output dtype")
    b = None
    if bias is not None:
        b = bias.to(device=dev, dtype=torch.bfloat16).contiguous()
        if b.numel() != rows:
            raise ValueError(f"radix_ops: bias has {b.numel()} entries, the tensor {rows} rows")
    _lib.call("dm_gemv", h.ptr, ct.c_void_p(x.data_ptr()), _DT[x.dtype], M,
              ct.c_void_p(b.data_ptr() if b is not None else 0), ct.c_void_p(out.data_ptr()), _DT[out_dtype],
              _stream(dev))
    return out


def gemv_fused(p: dict, x: torch.Tensor, bias, out_dtype=torch.bfloat16) -> torch.Tensor:
    """The M=1 arm: x [C] (bf16 or fp32) -> [1, R] in `out_dtype`, the bias
    (if any) added in fp32 before the single rounding."""
    return _run(p, x.reshape(1, -1), bias, out_dtype)


def gemv(p: dict, x: torch.Tensor) -> torch.Tensor:
    """The M=1 arm's fp32 [R] result, no bias."""
    return _run(p, x.reshape(1, -1), None, torch.float32).reshape(-1)


def gemv_mc(p: dict, x: torch.Tensor) -> torch.Tensor:
    """The multi-column arm: x [M, C] (bf16 or fp32), 1 <= M <= MC_MAX ->
    fp32 [M, R]; each row bitwise the M=1 arm's."""
    M = x.shape[0]
    if not 1 <= M <= MC_MAX:
        raise ValueError(f"radix gemv_mc: M={M} outside 1..{MC_MAX}")
    return _run(p, x, None, torch.float32)


def gemv_mc_fused(p: dict, x: torch.Tensor, bias, out_dtype) -> torch.Tensor:
    """gemv_mc with the epilogue fused: [M, R] in `out_dtype`, the bias added
    in fp32 before one rounding — the arithmetic of CompressedLinear._epilogue
    (swap.py:284-300) in the kernel."""
    return _run(p, x, bias, out_dtype)


def gemv_into(p: dict, x: torch.Tensor, bias, out: torch.Tensor) -> torch.Tensor:
    """gemv_mc_fused writing into a caller-owned [M, rows] tensor (bf16 or
    fp32): no allocation, so a chain of calls captures into one CUDA graph
    with static addresses."""
    return _run(p, x.reshape(-1, x.shape[-1]), bias, out.dtype, out)


def gemv_narrow(w: torch.Tensor, x: torch.Tensor, bias, block: int = 512, num_warps: int = 4) -> torch.Tensor:
    """NarrowLinear's forward: x [M, C] (bf16 or fp32) against the row-major
    bf16 weight w [R, C] -> [M, R] in x's dtype, the bias added in fp32
    before the one rounding. `block` / `num_warps` are the reference's
    launch knobs, accepted for the signature; this kernel sizes itself."""
    M, C = x.shape
    if not 1 <= M <= MC_MAX:
        raise ValueError(f"gemv_narrow: M={M} outside 1..{MC_MAX}")
    return gemv_raw(w, x, bias, x.dtype)


def gemv_raw(w: torch.Tensor, x: torch.Tensor, bias, out_dtype) -> torch.Tensor:
    """Raw bf16 GEMV for 1 <= M <= MC_MAX rows (the raw lm_head's one-row call
    and the narrow Linears)."""
    if w.dtype != torch.bfloat16 or w.dim() != 2:
        raise TypeError("gemv_raw: the weight must be a 2-D bf16 tensor")
    dev = w.device
    x = _check_x(x.reshape(-1, w.shape[1]), w.shape[1], dev)
    M = x.shape[0]
    if not 1 <= M <= MC_MAX:
        raise ValueError(f"gemv_narrow: M={M} outside 1..{MC_MAX}")
    w = w.contiguous()
    R, C = w.shape
    out = torch.empty((M, R), dtype=out_dtype, device=dev)
    b = bias.to(device=dev, dtype=torch.bfloat16).contiguous() if bias is not None else None
    _lib.call("dm_gemv_raw", ct.c_void_p(w.data_ptr()), R, C, ct.c_void_p(x.data_ptr()), _DT[x.dtype], M,
              ct.c_void_p(b.data_ptr() if b is not None else 0), ct.c_void_p(out.data_ptr()), _DT[out_dtype],
              _stream(dev))
    return out


def prefill(p: dict, x: torch.Tensor, bias, out_dtype=torch.bfloat16) -> torch.Tensor:
    """The prefill arm for a sip tensor: x [M, C] bf16 -> [M, R] in
    `out_dtype`, the weights decoded into shared memory and contracted on the
    tensor cores (tcgen05, fp32 accumulate), the bias added in fp32 before
    the one rounding — the dense arm's arithmetic (radix_kernel_gpu.py:
    615-636) without the decoded weight in HBM."""
    h = _handle(p)
    dev = h.torch_device
    x = _check_x(x.reshape(-1, h.info.C), h.info.C, dev)
    if x.dtype != torch.bfloat16:
        x = x.to(torch.bfloat16)
    if x.data_ptr() % 16:
        x = x.clone()  # the kernel's TMA reads the activations from a 16-byte aligned base
    if out_dtype not in _DT:
        raise TypeError(f"radix_ops: output dtype must be bf16 or fp32, not {out_dtype}")
    M = x.shape[0]
    rows = h.info.rows
    out = torch.empty((M, rows), dtype=out_dtype, device=dev)
    b = None
    if bias is not None:
        b = bias.to(device=dev, dtype=torch.bfloat16).contiguous()
    nbytes = int(_lib.lib().dm_prefill_workspace_bytes(h.ptr, M))
    work = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=dev)
    _lib.call("dm_prefill", h.ptr, ct.c_void_p(x.data_ptr()), M, ct.c_void_p(b.data_ptr() if b is not None else 0),
              ct.c_void_p(out.data_ptr()), _DT[out_dtype], ct.c_void_p(work.data_ptr()), work.numel(), _stream(dev))
    return out


def decode_bits(p: dict, num_warps: int = 2) -> torch.Tensor:
    """Every block decoded to the original uint16 bit patterns [R, C]."""
    h = _handle(p)
    out = torch.empty((h.info.rows, h.info.C), dtype=torch.uint16, device=h.torch_device)
    _lib.call("dm_decode", h.ptr, ct.c_void_p(out.data_ptr()), _stream(h.torch_device))
    return out


def decode_weight(p: dict) -> torch.Tensor:
    """The transient bf16 weight [R, C] (the dense arm's F.linear operand)."""
    return decode_bits(p).view(torch.bfloat16)


def prepare_schedule(data: torch.Tensor, offsets: torch.Tensor, C: int, widths, B: int, nblocks: int):
    """The gulp profile's per-block stream lengths (uint16 per block) over the
    pack's original payload and directory, on the device."""
    if data.device.type != "cuda":
        raise ValueError("prepare_schedule: the payload must be on a CUDA device")
    sched = torch.empty(nblocks, dtype=torch.uint16, device=data.device)
    d = data.contiguous()
    o = offsets.to(device=data.device).contiguous()
    w = (ct.c_int32 * len(widths))(*[int(v) for v in widths])
    _lib.call("dm_prepare_schedule", ct.c_void_p(d.data_ptr()), d.numel(), ct.c_void_p(o.data_ptr()), int(C), w,
              len(widths), int(B), int(nblocks), ct.c_void_p(sched.data_ptr()), _stream(data.device))
    return sched


def read_bytes(p: dict) -> int:
    """Bytes one GEMV/MC call streams (the reference's count): the payload
    NW words, the directory, the padded lookup tables and (gulp) the
    schedule."""
    return int(_handle(p).info.read_bytes)


def launch_of(p: dict) -> dict:
    return p.get("rx_launch") or {}
