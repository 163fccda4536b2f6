"""ctypes binding of libdrinkme_b200.so (the C ABI of include/drinkme_b200.h).

The library is built in-tree (``python -m drinkme_b200.build``). There is no
fallback: a missing library, or a call that fails, raises.
"""
from __future__ import annotations

import ctypes as ct
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libdrinkme_b200.so")

DM_OK, DM_EINVAL, DM_ECUDA, DM_EDEVICE, DM_ENOMEM = 0, 1, 2, 3, 4
DM_BF16, DM_F32 = 0, 1
DM_MC_MAX = 8
DM_MAX_RANKS = 8

EXPORTS = ("dm_version", "dm_tensor_create", "dm_tensor_create_multi", "dm_tensor_clone", "dm_tensor_destroy", "dm_tensor_get_info", "dm_gemv",
           "dm_gemv_noalloc", "dm_decode",
           "dm_prepare_schedule", "dm_gemv_raw", "dm_pack_plan", "dm_pack_encode", "dm_pack_plan_device", "dm_pack_encode_device", "dm_decode_pack", "dm_step_add_rmsnorm", "dm_step_qk_rope_cache", "dm_step_attention_workspace_bytes", "dm_step_attention", "dm_step_silu_mul", "dm_step_attention_block_workspace_bytes", "dm_step_attention_block", "dm_tensor_check",
           "dm_prefill", "dm_prefill_workspace_bytes", "dm_gemv_gather", "dm_tensor_set_launch", "dm_gemv_plan", "dm_ipc_handle", "dm_ipc_open", "dm_ipc_close", "dm_device_alloc", "dm_device_free",
           "dm_chain_create", "dm_chain_run", "dm_chain_destroy")


class DrinkmeError(RuntimeError):
    """A C-ABI call failed; .status is the DM_* code."""

    def __init__(self, status: int, msg: str):
        super().__init__(msg)
        self.status = status


class TensorInfo(ct.Structure):
    _fields_ = [("R", ct.c_int64), ("C", ct.c_int64), ("row_begin", ct.c_int64), ("rows", ct.c_int64),
                ("block_size", ct.c_int32), ("nwidths", ct.c_int32), ("widths", ct.c_int32 * 8),
                ("nblocks", ct.c_int64), ("payload_words", ct.c_int64), ("read_bytes", ct.c_int64),
                ("resident_bytes", ct.c_int64), ("fast_path", ct.c_int32), ("device", ct.c_int32),
                ("device_bytes_per_call", ct.c_int64), ("layout_ptr", ct.c_uint64), ("layout_bytes", ct.c_int64)]


class PackPart(ct.Structure):
    """dm_pack_part: one pack (or row range of one) of a fused tensor."""
    _fields_ = [("host_palette", ct.c_void_p), ("npalette", ct.c_size_t), ("host_offsets", ct.c_void_p),
                ("noffsets", ct.c_size_t), ("host_data", ct.c_void_p), ("nwords", ct.c_size_t),
                ("R", ct.c_int64), ("C", ct.c_int64), ("host_widths", ct.c_void_p), ("nwidths", ct.c_int32),
                ("block_size", ct.c_int32), ("row_begin", ct.c_int64), ("row_end", ct.c_int64)]


class Launch(ct.Structure):
    """dm_launch: a sip tensor's launch knobs."""
    _fields_ = [("slots", ct.c_int32), ("split", ct.c_int32), ("skew", ct.c_int32), ("resident", ct.c_int32),
                ("prefetch", ct.c_int32)]


class LaunchPlan(ct.Structure):
    """dm_launch_plan: what a GEMV launch would be."""
    _fields_ = [("grid", ct.c_int32), ("split", ct.c_int32), ("slots", ct.c_int32), ("resident", ct.c_int32),
                ("smem_bytes", ct.c_int32), ("skew_step", ct.c_int32)]


class Gather(ct.Structure):
    """dm_gather: the fused NVLink output gather of one row-sharded linear."""
    _fields_ = [("world", ct.c_int32), ("rank", ct.c_int32), ("slot", ct.c_int64),
                ("peer_out", ct.c_void_p * DM_MAX_RANKS), ("peer_flags", ct.c_void_p * DM_MAX_RANKS),
                ("gen", ct.c_void_p), ("done", ct.c_void_p), ("wait_flags", ct.c_void_p), ("wait_gen", ct.c_void_p),
                ("abort", ct.c_void_p), ("wait_polls", ct.c_uint32)]


class ChainLink(ct.Structure):
    """dm_chain_link: one linear of a persistent chain launch."""
    _fields_ = [("t", ct.c_void_p), ("x", ct.c_void_p), ("bias", ct.c_void_p), ("g", Gather), ("wait", ct.c_int32)]


_LIB = None


def lib():
    """The loaded library; raises when it was not built."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"drinkme_b200: the CUDA library is not built ({LIB_PATH}); "
                              "run `python -m drinkme_b200.build`")
        L = ct.CDLL(LIB_PATH)
        p, i32, i64, sz = ct.c_void_p, ct.c_int32, ct.c_int64, ct.c_size_t
        cp = ct.c_char_p
        L.dm_version.argtypes = []
        L.dm_tensor_create.argtypes = [p, sz, p, sz, p, sz, i64, i64, p, i32, i32, i64, i64, i32, ct.POINTER(p), cp, sz]
        L.dm_tensor_create_multi.argtypes = [ct.POINTER(PackPart), i32, i32, ct.POINTER(p), cp, sz]
        L.dm_tensor_clone.argtypes = [p, ct.POINTER(p), cp, sz]
        L.dm_tensor_destroy.argtypes = [p]
        L.dm_tensor_get_info.argtypes = [p, ct.POINTER(TensorInfo)]
        L.dm_gemv.argtypes = [p, p, i32, i64, p, p, i32, p, cp, sz]
        L.dm_gemv_noalloc.argtypes = [p, p, i32, i64, p, p, i32, p, cp, sz]
        L.dm_decode.argtypes = [p, p, p, cp, sz]
        L.dm_prepare_schedule.argtypes = [p, sz, p, i64, p, i32, i32, i64, p, p, cp, sz]
        L.dm_gemv_raw.argtypes = [p, i64, i64, p, i32, i64, p, p, i32, p, cp, sz]
        L.dm_pack_plan.argtypes = [p, i64, i64, p, i32, i32, i32, p, p, ct.POINTER(ct.c_uint64), cp, sz]
        L.dm_pack_encode.argtypes = [p, i64, i64, p, i32, i32, i32, p, p, p, ct.c_uint64, cp, sz]
        L.dm_decode_pack.argtypes = [p, sz, p, sz, sz, i64, i64, p, i32, i32, p, p, p, p, cp, sz]
        L.dm_pack_plan_device.argtypes = [p, i64, i64, p, i32, i32, p, p, ct.POINTER(ct.c_uint64), p, cp, sz]
        L.dm_pack_encode_device.argtypes = [p, i64, i64, p, i32, i32, p, p, p, ct.c_uint64, p, cp, sz]
        L.dm_step_add_rmsnorm.argtypes = [p, p, p, p, i64, ct.c_float, p, cp, sz]
        L.dm_step_qk_rope_cache.argtypes = [p, p, p, p, p, p, p, p, p, i32, i32, i32, ct.c_float, p, cp, sz]
        L.dm_step_attention_workspace_bytes.argtypes = [i32, i32, i64]
        L.dm_step_attention.argtypes = [p, p, p, p, i64, p, p, i32, i32, i32, p, cp, sz]
        L.dm_step_silu_mul.argtypes = [p, p, i64, p, cp, sz]
        L.dm_step_attention_block_workspace_bytes.argtypes = [i32, i32, i32, i64]
        L.dm_step_attention_block.argtypes = [p, p, p, p, p, p, p, p, i64, p, p, i32, i32, i32, ct.c_float, p, cp, sz]
        L.dm_tensor_check.argtypes = [p, ct.POINTER(ct.c_int32), cp, sz]
        L.dm_prefill.argtypes = [p, p, i64, p, p, i32, p, i64, p, cp, sz]
        L.dm_prefill_workspace_bytes.argtypes = [p, i64]
        L.dm_gemv_gather.argtypes = [p, p, i64, p, i32, ct.POINTER(Gather), p, cp, sz]
        L.dm_ipc_handle.argtypes = [p, p, cp, sz]
        L.dm_ipc_open.argtypes = [p, i32, ct.POINTER(p), cp, sz]
        L.dm_ipc_close.argtypes = [p, cp, sz]
        L.dm_device_alloc.argtypes = [i32, sz, ct.POINTER(p), cp, sz]
        L.dm_device_free.argtypes = [p, cp, sz]
        L.dm_chain_create.argtypes = [ct.POINTER(ChainLink), i32, i64, i32, ct.POINTER(p), cp, sz]
        L.dm_chain_run.argtypes = [p, p, cp, sz]
        L.dm_chain_destroy.argtypes = [p, cp, sz]
        L.dm_tensor_set_launch.argtypes = [p, ct.POINTER(Launch), cp, sz]
        L.dm_gemv_plan.argtypes = [p, i64, i32, ct.POINTER(LaunchPlan), cp, sz]
        for name in EXPORTS:
            getattr(L, name).restype = ct.c_int
        L.dm_prefill_workspace_bytes.restype = ct.c_int64
        L.dm_step_attention_workspace_bytes.restype = ct.c_int64
        L.dm_step_attention_block_workspace_bytes.restype = ct.c_int64
        _LIB = L
    return _LIB


def call(fn: str, *args) -> None:
    """Call an entry point with the (err, err_len) tail appended; raise on a
    nonzero status (ValueError for DM_EINVAL, DrinkmeError otherwise)."""
    err = ct.create_string_buffer(1024)
    rc = getattr(lib(), fn)(*args, err, 1024)
    if rc != DM_OK:
        msg = err.value.decode(errors="replace") or f"{fn} failed with status {rc}"
        if rc == DM_EINVAL:
            raise ValueError(msg)
        raise DrinkmeError(rc, msg)
