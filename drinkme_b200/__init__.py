"""drinkme_b200 — drinkme's radix decode + linear hot path, native on B200 (sm_100a).

The packed BF16 weights of a drinkme pack (pack format 1, profiles sip and
gulp) are decoded inside hand-written CUDA kernels and contracted with the
activations there: the batch-1 GEMV, the 2..8-row narrow linear of MTP
verification, and (next) the prefill GEMM. Python drives the kernels through
the C ABI of ``libdrinkme_b200.so`` (include/drinkme_b200.h); the modules keep
the reference's operator interface (``radix_ops``, ``swap``).
"""
from __future__ import annotations

from .ops import MC_MAX  # noqa: F401

__all__ = ["MC_MAX", "codec", "radix_ops", "swap", "radix_schedule", "registry", "shard"]
__version__ = "0.1.0"
