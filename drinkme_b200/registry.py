"""The capability registry — the reference's codec/registry.py
(src/drinkme/codec/registry.py:81-153) with the B200 kernel family.

Key: (tensor_codec, layout, op, kernel). ``CUDA_SM100`` is this package's
kernel family (libdrinkme_b200.so); a row is True only where a gate passes:
the -m gpu parity tests (tests/test_gpu_parity.py) for DENSE, GEMV and MC.
The CPU column says False everywhere: this package has no CPU route (the
reference's CPU path is test infrastructure here, in oracle/).
"""
from __future__ import annotations

DENSE, GEMV, MC, ROW_SUBSET = "dense", "gemv", "mc", "row_subset"
OPS = (DENSE, GEMV, MC, ROW_SUBSET)
CUDA_SM100, CPU = "cuda_sm100", "cpu"
KERNELS = (CUDA_SM100, CPU)
RADIX, RAW, UNKNOWN = "radix", "raw", "unknown"
FORMATS = ((RADIX, 0), (RAW, 0))

TABLE: dict[tuple[str, int, str, str], bool] = {
    # radix: tests/test_gpu_parity.py — every bf16 pattern decodes exactly at
    # every profile and block size; GEMV and MC within the float64 bound
    # (2e-6 |x|.|W| + 1e-7) and 1e-3 of the reference's kernels
    (RADIX, 0, DENSE, CUDA_SM100): True,
    (RADIX, 0, GEMV, CUDA_SM100): True,
    (RADIX, 0, MC, CUDA_SM100): True,
    (RADIX, 0, ROW_SUBSET, CUDA_SM100): False,
    (RADIX, 0, DENSE, CPU): False,
    (RADIX, 0, GEMV, CPU): False,
    (RADIX, 0, MC, CPU): False,
    (RADIX, 0, ROW_SUBSET, CPU): False,
    # raw fallback: the raw GEMV (dm_gemv_raw) for M <= MC_MAX, cuBLAS above
    (RAW, 0, DENSE, CUDA_SM100): True,
    (RAW, 0, GEMV, CUDA_SM100): True,
    (RAW, 0, MC, CUDA_SM100): True,
    (RAW, 0, ROW_SUBSET, CUDA_SM100): False,
    (RAW, 0, DENSE, CPU): False,
    (RAW, 0, GEMV, CPU): False,
    (RAW, 0, MC, CPU): False,
    (RAW, 0, ROW_SUBSET, CPU): False,
}

_OP_NAMES = {DENSE: "dense decode", GEMV: "M=1 GEMV", MC: "multi-column GEMV",
             ROW_SUBSET: "row-subset (draft-vocab) projection"}


def _codec_key(tensor_codec):
    return tensor_codec if tensor_codec in (RADIX, RAW) else UNKNOWN


def supported(tensor_codec, layout: int, op: str, kernel: str) -> bool:
    return TABLE.get((_codec_key(tensor_codec), int(layout), op, kernel), False)


def describe(tensor_codec, layout: int) -> str:
    if tensor_codec == RADIX:
        return "radix (exponent tiers, literal sign/mantissa, 1024-weight blocks)"
    if tensor_codec == RAW:
        return "raw (bf16 bits verbatim — the radix fallback)"
    return f"unknown tensor kind {tensor_codec!r} layout-{int(layout)} (no codec named)"


def unsupported_note(tensor_codec, layout: int, op: str, kernel: str) -> str:
    known = (_codec_key(tensor_codec), int(layout), op, kernel) in TABLE
    return (f"the {_OP_NAMES.get(op, op)} has no {kernel} kernel for a {describe(tensor_codec, layout)} pack "
            f"tensor ({'unsupported' if known else 'unknown combination'} in drinkme_b200/registry.py)")


def kernel_of(device) -> str:
    import torch

    return CPU if torch.device(device).type == "cpu" else CUDA_SM100


def of_pack(p: dict) -> tuple:
    if p.get("codec") == RADIX:
        return RADIX, 0
    if p.get("codec") == RAW:
        return RAW, 0
    return UNKNOWN, int(p.get("layout", 0))
