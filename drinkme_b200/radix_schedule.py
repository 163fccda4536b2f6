"""The per-tensor launch schedule of the sm_100a sip kernels — this package's
counterpart of the reference's radix_schedule (src/drinkme/codec/
radix_schedule.py), keyed the same way and overridden through the same
variable, with the knobs these kernels really have.

The reference's rows pick Triton knobs (blocks per program, warps) per (box
class, profile family, shape class). The sm_100a GEMV has a fixed CTA shape
(one CTA per SM: a producer warp, four groups of four consumer warps and an
epilogue warp) and is tuned by four launch knobs instead, which reach the
kernel through dm_tensor_set_launch (include/drinkme_b200.h):

  slots     staging slots of the unit ring, 1..6; 0 = the measured rule
            (five, six at M = 1 for tensors of 8+ block columns)
  split     "auto" (cost rule: stream-K unless whole tiles keep the busiest
            CTA lighter), "stream" (stream-K over units), "tiles" (whole
            16-row tiles per CTA)
  skew      stream-K: how many units fewer than the average the last CTA to
            be dispatched gets (0..64; 4 measured best)
  resident  the most block columns whose activations stay resident in
            shared memory for the whole launch (0..16; 16 measured: wider
            tensors stage activations with every unit)

Slots and residency change only how data is staged: results are the same
bits. Split and skew change which CTA sums which units, so results may move
within the fp32-accumulation bound.

The rows below were measured on B200 with the per-launch CUDA-graph timing of
bench.py (Qwen3-8B and 32B shapes). Shape classes (radix_schedule.py:
351-362): head R >= 32768, narrow R <= 1024, long NB >= 8, wide R >= 8192,
else square. Families (365-370): two tiers -> "sip", three or more ->
"scheduled" (gulp and balanced packs with whole 1024-weight blocks are
re-encoded as sip by the loader, so they run these rows too; others run the
general kernel, which has no knobs).

DRINKME_RADIX_SCHEDULE (the reference's grammar, radix_schedule.py:372-417):
"table" (default), "spike" (the most conservative launch: whole tiles, two
slots, no residency), "key=value,..." over the keys above, a JSON object
{class: {key: value}} or "@file" holding one.
"""
from __future__ import annotations

import functools
import json
import os
from dataclasses import asdict, dataclass

CLASSES = ("head", "narrow", "long", "wide", "square")
FAMILIES = ("sip", "scheduled")
BOX_CLASSES = ("b200",)
SPLITS = {"auto": 0, "stream": 1, "tiles": 2}
KEYS = ("slots", "split", "skew", "resident")

# the measured defaults (sip.cu: resident_slots, the cost rule, kSkewUnits,
# kMaxResidentCols); a row differs from them where a class measured better
_DEFAULT = dict(slots=0, split="auto", skew=4, resident=16)
SPIKE = dict(slots=2, split="tiles", skew=0, resident=0)
TABLES = {"b200": {fam: {cls: dict(_DEFAULT) for cls in CLASSES} for fam in FAMILIES}}
KERNELS = {"sip": "sip-mma-sm100a", "scheduled": "sip-mma-sm100a"}


@dataclass(frozen=True)
class Launch:
    slots: int
    split: str
    skew: int
    resident: int
    shape_class: str
    family: str
    box_class: str
    source: str
    kernel: str

    def as_dict(self) -> dict:
        return asdict(self)

    def knobs(self) -> tuple[int, int, int, int]:
        """(slots, split code, skew, resident): dm_launch's fields."""
        return self.slots, SPLITS[self.split], self.skew, self.resident

    def describe(self) -> str:
        s = "rule" if self.slots == 0 else str(self.slots)
        return f"slots {s} split {self.split} skew {self.skew} resident {self.resident} [{self.kernel}]"


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
    if type(cfg["slots"]) is not int or not 0 <= cfg["slots"] <= 6:
        raise ValueError("radix schedule: slots must be 0 (the measured rule) or 1..6")
    if cfg["split"] not in SPLITS:
        raise ValueError(f"radix schedule: split must be one of {', '.join(SPLITS)}")
    if type(cfg["skew"]) is not int or not 0 <= cfg["skew"] <= 64:
        raise ValueError("radix schedule: skew must be 0..64")
    if type(cfg["resident"]) is not int or not 0 <= cfg["resident"] <= 16:
        raise ValueError("radix schedule: resident must be 0..16")


def _value(key: str, value):
    if key == "split":
        return str(value).strip()
    if key == "slots" and str(value).strip() in ("rule", "auto"):
        return 0
    return int(value)


def _parse_override(spec: str) -> dict:
    out = {}
    for item in spec.split(","):
        item = item.strip()
        if not item:
            continue
        key, _, value = item.partition("=")
        key = key.strip()
        if key not in KEYS:
            raise ValueError(f"DRINKME_RADIX_SCHEDULE: unknown key {key!r} in {spec!r} (keys: {', '.join(KEYS)}; "
                             "tiles / warps are the reference's Triton knobs, which this kernel does not have)")
        out[key] = _value(key, value)
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
            if key not in KEYS:
                raise ValueError(f"DRINKME_RADIX_SCHEDULE: unknown key {key!r} for class {cls!r}")
            cfg[key] = _value(key, value)
        _validate({**_DEFAULT, **cfg})
        out[cls] = cfg
    return out


def select(R: int, C: int, block_size: int = 1024, widths=(3, 8), override: str | None = None) -> Launch:
    """The launch of an (R, C) radix tensor: the b200 table's row for its
    (family, shape class), or the DRINKME_RADIX_SCHEDULE override."""
    cls, fam, box = shape_class(R, C, block_size), family(widths), "b200"
    kernel = KERNELS[fam] if int(block_size) == 1024 and int(C) % 1024 == 0 else "generic-sm100a"
    spec = os.environ.get("DRINKME_RADIX_SCHEDULE", "table") if override is None else override
    spec = (spec or "table").strip()
    if spec in ("table", "table=b200"):
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
_validate(SPIKE)
