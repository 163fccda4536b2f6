"""The CPU oracle is pinned before it is trusted: against the golden vectors
the reference produced (tests/golden/make_golden.py), against an independent
numpy restatement, and against the reference's own native codec compiled
from its sources (oracle/_ref, when built)."""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

from conftest import GOLDEN, ROOT, all_patterns, pack_of, radix_names

sys.path.insert(0, ROOT)
from oracle import oracle  # noqa: E402


def test_oracle_decodes_every_golden_pack_bit_exact(golden):
    z, pins = golden
    for name in radix_names(pins):
        p = pack_of(z, pins, name)
        assert np.array_equal(oracle.decode(p), z[f"{name}/bits"]), name


def test_numpy_restatement_agrees_with_the_c_oracle(golden):
    z, pins = golden
    for name in radix_names(pins):
        p = pack_of(z, pins, name)
        assert np.array_equal(oracle.decode_numpy(p), oracle.decode(p)), name


def test_oracle_schedule_matches_the_reference_schedule(golden):
    z, pins = golden
    seen = 0
    for name in radix_names(pins):
        p = pack_of(z, pins, name)
        s = oracle.schedule(p)
        key = f"{name}/schedule"
        if key in z.files:
            assert np.array_equal(s, z[key]), name
            seen += 1
        else:
            assert s is None
    assert seen >= 10


def test_reference_native_decoder_agrees(golden):
    if oracle.reference_native() is None:
        pytest.skip("the reference's native codec is not built (oracle/_ref)")
    z, pins = golden
    for name in radix_names(pins):
        p = pack_of(z, pins, name)
        if p["block_size"] != 1024:
            continue
        assert np.array_equal(oracle.reference_decode(p), z[f"{name}/bits"]), name


def test_oracle_linear_bounds_the_reference_kernels(golden):
    """The reference's own fp32 GEMV (its Triton kernels, interpreted) lies
    inside the float64 gate this oracle computes — the gate the CUDA path
    must also pass (bench/radix_gemv_bitpin.py:182)."""
    z, pins = golden
    for name in radix_names(pins):
        if f"{name}/gemv_bf16x" not in z.files:
            continue
        bits = z[f"{name}/bits"]
        xb = z[f"{name}/x_bf16"].astype(np.uint32) << 16
        x = xb.view(np.float32)
        y, bound = oracle.gemv_bound(x[:1], bits)
        assert np.all(np.abs(z[f"{name}/gemv_bf16x"].astype(np.float64) - y[0]) <= bound[0]), name
        y8, b8 = oracle.gemv_bound(x[:8], bits)
        assert np.all(np.abs(z[f"{name}/mc8_bf16x"].astype(np.float64) - y8) <= b8), name


@pytest.mark.parametrize("profile", ["sip", "balanced", "gulp"])
def test_oracle_validate_messages(golden, profile):
    z, pins = golden
    p = pack_of(z, pins, f"{profile}_normal_16x4096")
    oracle.validate(p)
    bad = dict(p, rx_offsets=p["rx_offsets"][:-1])
    with pytest.raises(oracle.OracleError, match="offsets"):
        oracle.validate(bad)
    off = p["rx_offsets"].copy()
    off[1] = 1
    with pytest.raises(oracle.OracleError, match="fewer than the"):
        oracle.validate(dict(p, rx_offsets=off))
    with pytest.raises(oracle.OracleError, match="palette"):
        oracle.validate(dict(p, rx_palette=np.zeros_like(p["rx_palette"])))


def test_oracle_refuses_a_block_short_of_its_terminal_stream():
    """radix.py test: a block cut after its fixed streams but short of its
    terminal exponents passes validate and the strict decoder refuses it
    ('truncated radix stream', tests/test_radix.py:61-74)."""
    from drinkme_b200 import codec

    bits = np.full((4, 1024), 0x3F80, np.uint16)
    bits[1, 100:140] = np.arange(40, dtype=np.uint16) << 7
    pal, off, data = codec.encode_arrays(bits, (3, 8))
    p = {"rx_palette": pal, "rx_offsets": off, "rx_data": data, "R": 4, "C": 1024, "widths": [3, 8],
         "block_size": 1024}
    fewest, _ = oracle.word_bounds(1024, (3, 8))
    terminal = int(off[2] - off[1] - fewest)
    assert terminal == 9
    off2 = off.copy()
    off2[2:] -= terminal
    cut = dict(p, rx_offsets=off2, rx_data=np.delete(data, np.s_[off2[2]:off2[2] + terminal]))
    oracle.validate(cut)
    with pytest.raises(oracle.OracleError, match="truncated radix stream"):
        oracle.decode(cut)


def test_all_patterns_round_trip_through_the_oracle():
    from drinkme_b200 import codec

    ex = all_patterns()
    for prof, widths in codec.PROFILES.items():
        for block in (32, 1024):
            pal, off, data = codec.encode_arrays(ex, widths, block)
            p = {"rx_palette": pal, "rx_offsets": off, "rx_data": data, "R": 512, "C": 513,
                 "widths": list(widths), "block_size": block}
            assert np.array_equal(oracle.decode(p), ex), (prof, block)


def test_golden_files_exist():
    assert os.path.exists(os.path.join(GOLDEN, "packs.npz"))
    assert os.path.exists(os.path.join(GOLDEN, "pins.json"))
