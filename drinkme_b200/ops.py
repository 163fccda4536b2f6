"""Constants the operator side reads on any machine: MC_MAX, the widest
activation batch one multi-column call serves (the reference's
src/drinkme/codec/ops.py:19 and the C ABI's DM_MC_MAX)."""
from __future__ import annotations

MC_MAX = 8
