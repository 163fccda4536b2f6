"""The pack encoder on the GPU (dm_pack_plan_device / dm_pack_encode_device,
codec.encode_arrays_device) writes the reference's bytes: every golden pack,
the 65,536-pattern pins at every profile and block size, the config-1
down_proj pin, ragged shapes and widths of every tier count, and the same
raw-fallback decision as the host encoder (tests/test_encoder.py)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import all_patterns, pack_of, sha
from drinkme_b200 import codec, radix_ops, swap

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _dev(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits, dtype=np.uint16).view(np.int16)).to(DEV)


def _same(a, b):
    for x, y in zip(a, b):
        assert x.dtype == y.dtype and np.array_equal(x, y)


def test_every_golden_pack_on_the_gpu(golden):
    z, pins = golden
    for name, m in pins["packs"].items():
        bits = z[f"{name}/bits"]
        p = codec.pack_array_radix_device(_dev(bits), m["profile"], block_size=m["block_size"])
        if m.get("raw_fallback"):
            assert p is None, name
            continue
        ref = pack_of(z, pins, name)
        for k in ("rx_palette", "rx_offsets", "rx_data"):
            assert np.array_equal(p[k], ref[k]), (name, k)
        assert p["bpw"] == pytest.approx(m["bpw"])


@pytest.mark.parametrize("profile", ["sip", "balanced", "gulp"])
@pytest.mark.parametrize("block", [32, 1024])
def test_all_pattern_pins_on_the_gpu(golden, profile, block):
    _, pins = golden
    pal, off, data = codec.encode_arrays_device(_dev(all_patterns()), codec.PROFILES[profile], block)
    pin = pins["all_patterns"][f"{profile}/{block}"]
    assert sha(pal, off, data) == pin["sha256"]
    assert pal.tolist() == pin["palette"]


def test_config1_down_proj_pin_on_the_gpu(golden):
    """8B down_proj 4096 x 12288, N(0, 0.02) from seed 0,
    and the round trip through the loader and the GPU decode."""
    _, pins = golden
    g = torch.Generator().manual_seed(0)
    W = (torch.randn(4096, 12288, generator=g) * 0.02).to(torch.bfloat16)
    bits = W.view(torch.int16).to(DEV)
    for prof in ("sip", "gulp"):
        p = codec.pack_array_radix_device(bits, prof)
        pin = pins["config1"][prof]
        assert sha(p["rx_palette"], p["rx_offsets"], p["rx_data"]) == pin["sha256"], prof
        assert p["bpw"] == pytest.approx(pin["bpw"])
    rt = swap.to_device_radix(p, DEV)
    assert torch.equal(radix_ops.decode_bits(rt).view(torch.int16), bits)


@pytest.mark.parametrize("widths", [(3, 8), (2, 2, 4, 8), (1, 1, 1, 1, 1, 1, 1, 8), (8, 8), (4, 8), (1, 8)])
def test_ragged_shapes_and_tier_counts_match_the_host_encoder(widths):
    rng = np.random.default_rng(sum(widths))
    for (R, C), block in (((1, 31), 32), ((7, 33), 32), ((3, 1025), 1024), ((2, 4101), 4096), ((5, 3000), 256),
                          ((64, 2048), 1024)):
        e = np.clip(np.rint(rng.normal(120, 3 + len(widths), (R, C))), 0, 255).astype(np.uint16)
        bits = (e << 7) | rng.integers(0, 128, (R, C), dtype=np.uint16) | (rng.integers(0, 2, (R, C),
                                                                                         dtype=np.uint16) << 15)
        _same(codec.encode_arrays_device(_dev(bits), widths, block), codec.encode_arrays(bits, widths, block))


def test_raw_fallback_decision_matches_the_host():
    rng = np.random.default_rng(19)
    a = rng.integers(0, 65536, (128, 1024), dtype=np.uint16)
    assert codec.pack_array_radix_device(_dev(a), "sip") is None
    assert codec.pack_array_radix(a, "sip") is None


def test_refusals():
    with pytest.raises(ValueError):
        codec.encode_arrays_device(_dev(np.zeros((4, 1024), np.uint16)), (3, 8), 48)
    with pytest.raises(ValueError):
        codec.encode_arrays_device(_dev(np.zeros((4, 1024), np.uint16)), (9, 8), 1024)
    with pytest.raises(TypeError):
        codec.encode_arrays_device(np.zeros((4, 1024), np.uint16), (3, 8), 1024)


def test_decode_and_hash_rebuilds_the_source_file():
    """verify.rebuild_sha256: a file of raw bytes (a header), a sip tensor, a
    gulp tensor and a raw tensor hashes like the source bits; one changed
    weight changes the verdict."""
    import hashlib

    from drinkme_b200 import verify

    g = torch.Generator().manual_seed(3)
    Ws = [(torch.randn(r, c, generator=g) * 0.02).to(torch.bfloat16) for r, c in ((300, 4096), (64, 2048), (16, 512))]
    header = b"\x20\x00\x00\x00\x00\x00\x00\x00" + b'{"__metadata__":{"format":"pt"}}'
    parts = [header, codec.pack_weight_radix(Ws[0], "sip"), codec.pack_weight_radix(Ws[1], "gulp"),
             codec.raw_dict(codec.bits_of(Ws[2])), b"tail"]
    assert parts[1]["codec"] == "radix" and parts[2]["codec"] == "radix"
    want = hashlib.sha256()
    want.update(header)
    for W in Ws:
        want.update(codec.bits_of(W).tobytes())
    want.update(b"tail")
    got = verify.rebuild_sha256(parts, DEV)
    assert got["sha256"] == want.hexdigest()
    assert got["bytes"] == len(header) + sum(W.numel() * 2 for W in Ws) + 4
    assert verify.verify_parts(parts, want.hexdigest(), DEV) == "MATCH"
    W2 = Ws[0].clone()
    W2[7, 11] = -W2[7, 11] if float(W2[7, 11]) != 0 else 1.0
    parts[1] = codec.pack_weight_radix(W2, "sip")
    assert verify.verify_parts(parts, want.hexdigest(), DEV) == "MISMATCH"


def test_verify_files_in_parallel():
    import hashlib

    from drinkme_b200 import verify

    g = torch.Generator().manual_seed(4)
    files, wants = [], []
    for k in range(3):
        W = (torch.randn(64 + 16 * k, 2048, generator=g) * 0.02).to(torch.bfloat16)
        files.append([b"h%d" % k, codec.pack_weight_radix(W, "sip")])
        wants.append(hashlib.sha256(b"h%d" % k + codec.bits_of(W).tobytes()).hexdigest())
    out = verify.verify_files(zip(files, wants[:2] + ["0" * 64]), DEV, workers=3)
    assert [o["verdict"] for o in out] == ["MATCH", "MATCH", "MISMATCH"]
    assert out[2]["sha256"] == wants[2]


def test_decode_pack_as_stored(golden):
    """dm_decode_pack: every golden pack (every profile, block size and ragged
    shape) decoded on the GPU from its own arrays is its source bits; a
    directory that does not fit the words is refused with validate's message."""
    z, pins = golden
    for name, m in pins["packs"].items():
        if m.get("raw_fallback"):
            continue
        p = pack_of(z, pins, name)
        got = codec.decode_pack_device(p, DEV).cpu().numpy().view(np.uint16)
        assert np.array_equal(got, z[f"{name}/bits"]), name
    p = dict(pack_of(z, pins, "sip_normal_16x4096"))
    p["rx_offsets"] = p["rx_offsets"].copy()
    p["rx_offsets"][-1] += 7
    with pytest.raises(ValueError):
        codec.decode_pack_device(p, DEV)
