"""A device-resident radix tensor: the owner of one dm_tensor handle of the C
library (dm_tensor_create / dm_tensor_destroy)."""
from __future__ import annotations

import ctypes as ct

import numpy as np
import torch

from . import _lib


class RadixTensor:
    """Rows [row_begin, row_end) of a pack-format-1 radix tensor laid out on a
    CUDA device for the sm_100a kernels. Validation runs in the library
    (radix.validate's rules and messages); a malformed pack raises
    ValueError and allocates nothing."""

    def __init__(self, pack: dict, device, row_begin: int = 0, row_end: int | None = None):
        dev = torch.device(device)
        if dev.type != "cuda":
            raise ValueError(f"drinkme_b200 serves CUDA devices only, not {dev}")
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        pal = np.ascontiguousarray(pack["rx_palette"], dtype=np.uint8)
        off = np.ascontiguousarray(pack["rx_offsets"], dtype=np.uint32)
        data = np.ascontiguousarray(pack["rx_data"], dtype=np.uint32)
        if "NW" in pack:
            data = data[: int(pack["NW"])]
        widths = [int(w) for w in pack["widths"]]
        R, C = int(pack["R"]), int(pack["C"])
        row_end = R if row_end is None else int(row_end)
        w = (ct.c_int32 * len(widths))(*widths)
        handle = ct.c_void_p()
        _lib.call("dm_tensor_create", pal.ctypes.data_as(ct.c_void_p), pal.size, off.ctypes.data_as(ct.c_void_p),
                  off.size, data.ctypes.data_as(ct.c_void_p), data.size, R, C, w, len(widths),
                  int(pack["block_size"]), int(row_begin), row_end, int(dev.index), ct.byref(handle))
        self.ptr = handle
        self.torch_device = dev
        self.info = _lib.TensorInfo()
        _lib.lib().dm_tensor_get_info(self.ptr, ct.byref(self.info))
        self.palette = pal.copy()
        self.widths = tuple(widths)

    @classmethod
    def _wrap(cls, handle: ct.c_void_p, like: "RadixTensor") -> "RadixTensor":
        t = cls.__new__(cls)
        t.ptr = handle
        t.torch_device = like.torch_device
        t.info = _lib.TensorInfo()
        _lib.lib().dm_tensor_get_info(t.ptr, ct.byref(t.info))
        t.palette = like.palette
        t.widths = like.widths
        return t

    def clone(self) -> "RadixTensor":
        """A device-side copy in its own HBM (dm_tensor_clone)."""
        h = ct.c_void_p()
        _lib.call("dm_tensor_clone", self.ptr, ct.byref(h))
        return RadixTensor._wrap(h, self)

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
