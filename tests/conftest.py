"""Shared fixtures. `gpu` marks tests that need a B200 (run with -m gpu);
everything else runs on the CPU."""
from __future__ import annotations

import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (sm_100a); run with -m gpu")


def pytest_collection_modifyitems(config, items):
    try:
        import torch

        has_gpu = torch.cuda.is_available()
    except Exception:  # noqa: BLE001
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="needs a CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden():
    """(packs npz, pins json) generated from the reference by
    tests/golden/make_golden.py."""
    z = np.load(os.path.join(GOLDEN, "packs.npz"))
    with open(os.path.join(GOLDEN, "pins.json")) as f:
        pins = json.load(f)
    return z, pins


def pack_of(z, pins, name):
    """The pack dict of golden tensor `name` (None for a raw fallback)."""
    m = pins["packs"][name]
    if m.get("raw_fallback"):
        return None
    return {"rx_palette": z[f"{name}/palette"], "rx_offsets": z[f"{name}/offsets"], "rx_data": z[f"{name}/data"],
            "R": m["R"], "C": m["C"], "widths": m["widths"], "block_size": m["block_size"], "profile": m["profile"],
            "codec": "radix", "bpw": m["bpw"]}


def radix_names(pins):
    return [n for n, m in pins["packs"].items() if not m.get("raw_fallback")]


def sha(*arrays) -> str:
    import hashlib

    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


def all_patterns() -> np.ndarray:
    ex = np.zeros((512, 513), np.uint16)
    ex.flat[:65536] = np.arange(65536, dtype=np.uint16)
    return ex
