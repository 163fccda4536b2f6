"""The pack encoder (dm_pack_plan / dm_pack_encode) writes the reference's
bytes: every golden pack, the 65,536-pattern tensors at every profile and
block size (sha256 pins), the config-1 down_proj, and the raw fallback and
parameter refusals of radix.pack_array (tests/test_radix.py)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import all_patterns, pack_of, sha
from drinkme_b200 import codec


def test_every_golden_pack_is_reproduced_byte_for_byte(golden):
    z, pins = golden
    for name, m in pins["packs"].items():
        bits = z[f"{name}/bits"]
        p = codec.pack_array_radix(bits, m["profile"], block_size=m["block_size"])
        if m.get("raw_fallback"):
            assert p is None, name
            continue
        ref = pack_of(z, pins, name)
        for k in ("rx_palette", "rx_offsets", "rx_data"):
            assert np.array_equal(p[k], ref[k]), (name, k)
        assert p["bpw"] == pytest.approx(m["bpw"])


@pytest.mark.parametrize("profile", ["sip", "balanced", "gulp"])
@pytest.mark.parametrize("block", [32, 1024])
def test_all_pattern_pins(golden, profile, block):
    _, pins = golden
    pal, off, data = codec.encode_arrays(all_patterns(), codec.PROFILES[profile], block)
    pin = pins["all_patterns"][f"{profile}/{block}"]
    assert sha(pal, off, data) == pin["sha256"]
    assert pal.tolist() == pin["palette"]


def test_config1_down_proj_pin(golden):
    """8B down_proj 4096 x 12288, N(0, 0.02) from seed 0."""
    _, pins = golden
    g = torch.Generator().manual_seed(0)
    W = (torch.randn(4096, 12288, generator=g) * 0.02).to(torch.bfloat16)
    for prof in ("sip", "gulp"):
        p = codec.pack_weight_served(W, compression_profile=prof)
        pin = pins["config1"][prof]
        assert p["codec"] == "radix"
        assert sha(p["rx_palette"], p["rx_offsets"], p["rx_data"]) == pin["sha256"], prof
        assert int(p["rx_data"].size) == pin["words"]
        assert p["bpw"] == pytest.approx(pin["bpw"])


def test_incompressible_bits_fall_back_to_raw():
    rng = np.random.default_rng(19)
    a = rng.integers(0, 65536, (128, 1024), dtype=np.uint16)
    assert codec.pack_array_radix(a, "sip") is None
    w = torch.from_numpy(a.view(np.int16)).view(torch.bfloat16)
    p = codec.pack_weight_radix(w, "sip")
    assert p["codec"] == "raw" and np.array_equal(p["raw_bits"], a)


def test_ragged_rows_and_zero_escape_streams():
    for shape in [(1, 31), (7, 33), (3, 1023), (3, 1025), (2, 4101)]:
        for block in (32, 256, 1024, 4096):
            src = np.full((shape[0], shape[1] * 2), 0x3F81, np.uint16)[:, ::2]
            pal, off, data = codec.encode_arrays(src, (3, 8), block)
            from oracle import oracle

            p = {"rx_palette": pal, "rx_offsets": off, "rx_data": data, "R": shape[0], "C": shape[1],
                 "widths": [3, 8], "block_size": block}
            assert np.array_equal(oracle.decode(p), src)


@pytest.mark.parametrize("kwargs", [dict(block_size=31), dict(block_size=5000), dict(block_size=48)])
def test_invalid_block_sizes(kwargs):
    with pytest.raises(ValueError):
        codec.encode_arrays(np.zeros((4, 1024), np.uint16), (3, 8), kwargs["block_size"])


@pytest.mark.parametrize("widths", [(2,), (8, 8, 8), (2, 0, 8), (2, 4), (9, 8)])
def test_invalid_widths(widths):
    with pytest.raises(ValueError):
        codec.encode_arrays(np.zeros((4, 1024), np.uint16), widths, 1024)


def test_unknown_profile():
    with pytest.raises(ValueError):
        codec.pack_array_radix(np.zeros((4, 1024), np.uint16), "unknown")


def test_deterministic_bytes():
    a = np.tile(np.arange(65536, dtype=np.uint16), 4).reshape(256, 1024)
    a[:192] = 0x3F80
    one = codec.encode_arrays(a, (2, 2, 4, 8))
    two = codec.encode_arrays(a, (2, 2, 4, 8))
    for x, y in zip(one, two):
        assert np.array_equal(x, y)


def test_threads_do_not_change_bytes(golden):
    z, pins = golden
    bits = z["sip_tail_16x4096/bits"]
    one = codec.encode_arrays(bits, (3, 8), threads=1)
    many = codec.encode_arrays(bits, (3, 8), threads=8)
    for x, y in zip(one, many):
        assert np.array_equal(x, y)
