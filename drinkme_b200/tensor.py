"""A device-resident radix tensor: the owner of one dm_tensor handle of the C
library (dm_tensor_create / dm_tensor_destroy)."""
from __future__ import annotations

import ctypes as ct

import numpy as np
import torch

from . import _lib


def _cuda(device) -> torch.device:
    dev = torch.device(device)
    if dev.type != "cuda":
        raise ValueError(f"drinkme_b200 serves CUDA devices only, not {dev}")
    if dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    return dev


def device_view(ptr: int, shape, dtype: torch.dtype, device) -> torch.Tensor:
    """A torch tensor over device memory this package allocated (zero copy,
    through the CUDA array interface; bf16 travels as int16). The memory's
    owner must outlive the view."""
    code = {torch.bfloat16: "<i2", torch.float32: "<f4", torch.int32: "<i4", torch.uint8: "|u1"}[dtype]

    class _Raw:
        __cuda_array_interface__ = {"shape": tuple(shape), "typestr": code, "data": (int(ptr), False),
                                    "version": 3, "strides": None}

    t = torch.as_tensor(_Raw(), device=_cuda(device))
    return t.view(torch.bfloat16) if dtype == torch.bfloat16 else t


def _part(pack: dict, row_begin, row_end):
    """A dm_pack_part over a pack's host arrays, and the arrays to keep alive
    until the library has copied them."""
    pal = np.ascontiguousarray(pack["rx_palette"], dtype=np.uint8)
    off = np.ascontiguousarray(pack["rx_offsets"], dtype=np.uint32)
    data = np.ascontiguousarray(pack["rx_data"], dtype=np.uint32)
    if "NW" in pack:
        data = data[: int(pack["NW"])]
    widths = [int(w) for w in pack["widths"]]
    R, C = int(pack["R"]), int(pack["C"])
    w = (ct.c_int32 * len(widths))(*widths)
    part = _lib.PackPart(pal.ctypes.data, pal.size, off.ctypes.data, off.size, data.ctypes.data, data.size, R, C,
                         ct.cast(w, ct.c_void_p), len(widths), int(pack["block_size"]), int(row_begin or 0),
                         R if row_end is None else int(row_end))
    return part, (pal, off, data, w)


class RadixTensor:
    """Rows [row_begin, row_end) of a pack-format-1 radix tensor laid out on a
    CUDA device for the sm_100a kernels. Validation runs in the library
    (radix.validate's rules and messages); a malformed pack raises
    ValueError and allocates nothing."""

    def __init__(self, pack: dict, device, row_begin: int = 0, row_end: int | None = None):
        dev = _cuda(device)
        part, keep = _part(pack, row_begin, row_end)
        handle = ct.c_void_p()
        _lib.call("dm_tensor_create", part.host_palette, part.npalette, part.host_offsets, part.noffsets,
                  part.host_data, part.nwords, part.R, part.C, part.host_widths, part.nwidths, part.block_size,
                  part.row_begin, part.row_end, int(dev.index), ct.byref(handle))
        del keep
        self._init(handle, dev, np.ascontiguousarray(pack["rx_palette"], dtype=np.uint8).copy(),
                   tuple(int(w) for w in pack["widths"]))

    @classmethod
    def fused(cls, packs, device, ranges=None) -> "RadixTensor":
        """One handle over the rows of several packs sharing their columns
        (dm_tensor_create_multi): a GEMV on it yields [y_0 | y_1 | ...].
        `ranges` optionally gives each part's (row_begin, row_end)."""
        dev = _cuda(device)
        ranges = ranges or [(0, None)] * len(packs)
        if len(ranges) != len(packs):
            raise ValueError("RadixTensor.fused: one row range per pack")
        parts = (_lib.PackPart * len(packs))()
        keep = []
        for i, (pk, (r0, r1)) in enumerate(zip(packs, ranges)):
            parts[i], k = _part(pk, r0, r1)
            keep.append(k)
        handle = ct.c_void_p()
        _lib.call("dm_tensor_create_multi", parts, len(packs), int(dev.index), ct.byref(handle))
        del keep
        t = cls.__new__(cls)
        t._init(handle, dev, np.ascontiguousarray(packs[0]["rx_palette"], dtype=np.uint8).copy(),
                tuple(int(w) for w in packs[0]["widths"]))
        return t

    def _init(self, handle, dev, palette, widths) -> None:
        self.ptr = handle
        self.torch_device = dev
        self.info = _lib.TensorInfo()
        _lib.lib().dm_tensor_get_info(self.ptr, ct.byref(self.info))
        self.palette = palette
        self.widths = widths

    @classmethod
    def _wrap(cls, handle: ct.c_void_p, like: "RadixTensor") -> "RadixTensor":
        t = cls.__new__(cls)
        t._init(handle, like.torch_device, like.palette, like.widths)
        return t

    def clone(self) -> "RadixTensor":
        """A device-side copy in its own HBM (dm_tensor_clone)."""
        h = ct.c_void_p()
        _lib.call("dm_tensor_clone", self.ptr, ct.byref(h))
        return RadixTensor._wrap(h, self)

    def set_launch(self, slots: int = 0, split: int = 0, skew: int = -1, resident: int = -1,
                   prefetch: int = -1) -> None:
        """The sip kernels' launch knobs for this tensor (dm_tensor_set_launch;
        radix_schedule.Launch.knobs() gives them from the schedule table)."""
        _lib.call("dm_tensor_set_launch", self.ptr, ct.byref(_lib.Launch(slots, split, skew, resident, prefetch)))

    def plan(self, M: int = 1, dtype=torch.bfloat16) -> dict:
        """What a GEMV of M rows would launch (dm_gemv_plan): grid, split
        (1 stream-K, 2 tiles), slots, resident, smem_bytes, skew_step."""
        out = _lib.LaunchPlan()
        _lib.call("dm_gemv_plan", self.ptr, int(M), _lib.DM_F32 if dtype == torch.float32 else _lib.DM_BF16,
                  ct.byref(out))
        return {name: int(getattr(out, name)) for name, _ in _lib.LaunchPlan._fields_}

    def device_error(self) -> int:
        """The device error word (a bounded wait that gave up), read and cleared."""
        v = ct.c_int32()
        _lib.call("dm_tensor_check", self.ptr, ct.byref(v))
        return int(v.value)

    def close(self) -> None:
        if getattr(self, "ptr", None) is not None and self.ptr.value:
            _lib.lib().dm_tensor_destroy(self.ptr)
            self.ptr = ct.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass
