"""The per-tensor launch schedule — the reference's radix_schedule
(src/drinkme/codec/radix_schedule.py) with a ``b200`` box class.

The reference's table picks Triton knobs (blocks per program, warps) per
(box class, profile family, shape class), measured per GPU family. The
sm_100a kernels size themselves from the tensor and the shared-memory
budget (one CTA per SM, 8 consumer warps, 2-3 staged units each), so the
b200 rows name the kernel that serves each (family, class) and keep the
reference's fields for the boot log and for DRINKME_RADIX_SCHEDULE, whose
grammar (table | spike | tiles=..,warps=.. | {per-class json} | @file) is
parsed and validated the same way (radix_schedule.py:372-417, 461-489).

Shape classes (radix_schedule.py:351-362): head R >= 32768, narrow R <= 1024,
long NB >= 8, wide R >= 8192, else square. Families (365-370): two tiers ->
"sip", three or more -> "scheduled".
"""
from __future__ import annotations

import functools
import json
import os
from dataclasses import asdict, dataclass

SPIKE = dict(gemv_tiles=1, gemv_warps=2, mc_tiles=1, mc_warps=2)
CLASSES = ("head", "narrow", "long", "wide", "square")
FAMILIES = ("sip", "scheduled")
BOX_CLASSES = ("b200",)

# b200: gemv_tiles = 1 (one unit of 8 rows x 1 block per worker step, split-K
# across workers with a deterministic fixup), gemv_warps = 8 consumer warps.
_B200_ROW = dict(gemv_tiles=1, gemv_warps=8, mc_tiles=1, mc_warps=8)
TABLES = {"b200": {fam: {cls: dict(_B200_ROW) for cls in CLASSES} for fam in FAMILIES}}
KERNELS = {"sip": "sip-mma-sm100a", "scheduled": "generic-sm100a"}


@dataclass(frozen=True)
class Launch:
    gemv_tiles: int
    gemv_warps: int
    mc_tiles: int
    mc_warps: int
    shape_class: str
    family: str
    box_class: str
    source: str
    kernel: str

    def as_dict(self) -> dict:
        return asdict(self)

    def describe(self) -> str:
        g = "row" if self.gemv_tiles == 0 else str(self.gemv_tiles)
        m = "row" if self.mc_tiles == 0 else str(self.mc_tiles)
        return f"gemv {g}/w{self.gemv_warps} mc {m}/w{self.mc_warps} [{self.kernel}]"


def shape_class(R: int, C: int, block_size: int = 1024) -> str:
    nb = (int(C) + int(block_size) - 1) // int(block_size)
    R = int(R)
    if R >= 32768:
        return "head"
    if R <= 1024:
        return "narrow"
    if nb >= 8:
        return "long"
    if R >= 8192:
        return "wide"
    return "square"


def family(widths) -> str:
    return "sip" if len(tuple(widths)) <= 2 else "scheduled"


def _validate(cfg: dict) -> None:
    for key in ("gemv_tiles", "mc_tiles"):
        if type(cfg[key]) is not int or cfg[key] < 0:
            raise ValueError(f"radix schedule: {key} must be a non-negative int (0 = whole row)")
    for key in ("gemv_warps", "mc_warps"):
        if cfg[key] not in (1, 2, 4, 8):
            raise ValueError(f"radix schedule: {key} must be 1, 2, 4 or 8")


def _parse_override(spec: str) -> dict:
    out = {}
    for item in spec.split(","):
        item = item.strip()
        if not item:
            continue
        key, _, value = item.partition("=")
        key, value = key.strip(), value.strip()
        if key in ("tiles", "gemv_tiles"):
            out["gemv_tiles"] = 0 if value == "row" else int(value)
        elif key in ("warps", "gemv_warps"):
            out["gemv_warps"] = int(value)
        elif key == "mc_tiles":
            out["mc_tiles"] = 0 if value == "row" else int(value)
        elif key == "mc_warps":
            out["mc_warps"] = int(value)
        else:
            raise ValueError(f"DRINKME_RADIX_SCHEDULE: unknown key {key!r} in {spec!r}")
    return out


@functools.lru_cache(maxsize=8)
def _per_class_table(spec: str) -> dict:
    text = spec
    if spec.startswith("@"):
        with open(spec[1:]) as f:
            text = f.read()
    table = json.loads(text)
    if not isinstance(table, dict):
        raise ValueError("DRINKME_RADIX_SCHEDULE: a per-class table must be a JSON object")
    out = {}
    for cls, row in table.items():
        if cls not in CLASSES:
            raise ValueError(f"DRINKME_RADIX_SCHEDULE: unknown shape class {cls!r} (known: {sorted(CLASSES)})")
        if not isinstance(row, dict):
            raise ValueError(f"DRINKME_RADIX_SCHEDULE: class {cls!r} must map to an object")
        cfg = {}
        for key, value in row.items():
            if key not in SPIKE:
                raise ValueError(f"DRINKME_RADIX_SCHEDULE: unknown key {key!r} for class {cls!r}")
            cfg[key] = 0 if value == "row" else int(value)
        _validate({**SPIKE, **cfg})
        out[cls] = cfg
    return out


def select(R: int, C: int, block_size: int = 1024, widths=(3, 8), override: str | None = None) -> Launch:
    cls, fam, box = shape_class(R, C, block_size), family(widths), "b200"
    kernel = KERNELS[fam] if (fam == "sip" and int(block_size) == 1024 and int(C) % 1024 == 0) else "generic-sm100a"
    spec = os.environ.get("DRINKME_RADIX_SCHEDULE", "table") if override is None else override
    spec = (spec or "table").strip()
    if spec == "table" or spec == "table=b200":
        return Launch(**TABLES[box][fam][cls], shape_class=cls, family=fam, box_class=box, source="table",
                      kernel=kernel)
    if spec == "spike":
        return Launch(**SPIKE, shape_class=cls, family=fam, box_class=box, source="spike", kernel=kernel)
    cfg = dict(TABLES[box][fam][cls])
    if spec.startswith("{") or spec.startswith("@"):
        cfg.update(_per_class_table(spec).get(cls, {}))
    else:
        cfg.update(_parse_override(spec))
    _validate(cfg)
    return Launch(**cfg, shape_class=cls, family=fam, box_class=box, source="env", kernel=kernel)


for _rows in TABLES["b200"].values():
    for _cfg in _rows.values():
        _validate(_cfg)
