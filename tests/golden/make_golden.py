"""Generate the golden fixtures under tests/golden/ from the reference itself.

Run once in a container that holds the reference's sources (never on the GPU
box, never from a test):

    python tests/golden/make_golden.py --reference <reference checkout>

It imports the reference's Python package (``src/drinkme``), packs seeded
tensors with the reference's own packer, decodes them with the reference's
decoders, and runs the reference's Triton kernels under TRITON_INTERPRET=1
for kernel-order fp32 GEMV outputs. Outputs:

  packs.npz    small pack dicts (verbatim arrays), their source bits, the
               gulp schedules, activations and the reference's GEMV outputs
  pins.json    sha256 pins of larger packs (the 65,536-pattern tensors at
               every profile and block size; the config-1 down_proj), the
               reference's bpw and word counts, and the reference's CPU-route
               output for config 1
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


def normal_bits(R, C, seed, scale=0.02):
    import torch

    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(R, C, generator=g) * scale).to(torch.bfloat16)
    return w.view(torch.int16).numpy().view(np.uint16).copy()


def heavy_tail_bits(R, C, seed):
    """Finite bf16 bits whose exponents follow a geometric tail over 40
    values: every tier of every profile carries escapes, and most blocks
    have a terminal stream."""
    rng = np.random.default_rng(seed)
    k = np.arange(40)
    pk = 0.75 ** k
    exps = rng.choice(100 + k, size=(R, C), p=pk / pk.sum()).astype(np.uint16)
    bits = (exps << 7) | rng.integers(0, 128, (R, C), dtype=np.uint16)
    bits |= rng.integers(0, 2, (R, C), dtype=np.uint16) << 15
    return bits


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="the reference checkout (holds src/drinkme)")
    a = ap.parse_args()
    os.environ["TRITON_INTERPRET"] = "1"
    os.environ.setdefault("DRINKME_HOME", tempfile.mkdtemp(prefix="dmhome"))
    sys.path.insert(0, os.path.join(a.reference, "src"))
    import torch
    from drinkme.codec import radix, radix_ops, radix_pack as rp
    from drinkme.codec.pack import pack_weight_served
    from drinkme.codec.swap import make_module, to_device_radix

    packs = {}
    meta = {}

    def add(name, bits, profile, block=1024, gemv=True):
        if block == 1024:
            p = rp.pack_array_radix(bits, profile)
        else:
            rpk = radix.pack_array(bits, compression_profile=profile, block_size=block)
            p = None if rpk.raw else {"rx_palette": rpk.palette, "rx_offsets": rpk.offsets.astype(np.uint32),
                 "rx_data": rpk.data.astype(np.uint32), "R": bits.shape[0], "C": bits.shape[1],
                 "widths": list(rpk.widths), "block_size": block, "profile": profile, "codec": "radix"}
        if p is None:  # radix would expand it: the pack stores the raw fallback
            meta[name] = {"R": int(bits.shape[0]), "C": int(bits.shape[1]), "profile": profile,
                          "block_size": block, "raw_fallback": True}
            packs[f"{name}/bits"] = bits
            print(name, "raw fallback", flush=True)
            return
        back = rp.decode_back_radix(p) if block == 1024 else radix.decode(rp.as_radixpack(p))
        assert np.array_equal(back, bits)
        R, C = bits.shape
        d = {f"{name}/palette": p["rx_palette"], f"{name}/offsets": p["rx_offsets"],
             f"{name}/data": p["rx_data"], f"{name}/bits": bits}
        sched = rp.schedule_np(p)
        if sched is not None:
            d[f"{name}/schedule"] = sched
        m = {"R": R, "C": C, "widths": [int(w) for w in p["widths"]], "block_size": block,
             "profile": profile, "bpw": float(8.0 * (p["rx_palette"].nbytes + p["rx_offsets"].nbytes
                                                     + p["rx_data"].nbytes) / (R * C))}
        if gemv:
            rt = to_device_radix(p, "cpu")
            g = torch.Generator().manual_seed(1000 + len(packs))
            x32 = torch.randn(8, C, generator=g)
            xb = x32.to(torch.bfloat16)
            bias = torch.linspace(-0.1, 0.1, R).to(torch.bfloat16)
            d[f"{name}/x_bf16"] = xb.view(torch.int16).numpy().view(np.uint16)
            d[f"{name}/x_f32"] = x32[:1].numpy()
            d[f"{name}/bias_bf16"] = bias.view(torch.int16).numpy().view(np.uint16)
            d[f"{name}/gemv_bf16x"] = radix_ops.gemv(rt, xb[0]).numpy()
            d[f"{name}/gemv_f32x"] = radix_ops.gemv(rt, x32[0]).numpy()
            d[f"{name}/fused_bf16"] = radix_ops.gemv_fused(rt, xb[0], bias, torch.bfloat16).float().numpy()
            for M in (3, 8):
                d[f"{name}/mc{M}_bf16x"] = radix_ops.gemv_mc(rt, xb[:M]).numpy()
            if block == 1024:  # the native CPU decoder reads 1024-weight blocks only
                mod = make_module(p, bias, "cpu")
                d[f"{name}/cpu_route_bf16"] = mod(xb[:2]).float().numpy()
            m["gemv_launch"] = rt["rx_launch"]
        packs.update(d)
        meta[name] = m
        print(name, m["bpw"], flush=True)

    # small ragged shapes (bench/radix_gemv_bitpin.py RAGGED) and
    # production-like rows, at every profile
    for prof in ("sip", "balanced", "gulp"):
        for shape in ((1, 1), (7, 33), (3, 1025), (17, 3079), (129, 260)):
            add(f"{prof}_tail_{shape[0]}x{shape[1]}", heavy_tail_bits(*shape, seed=shape[0] * 31 + shape[1]), prof)
        add(f"{prof}_normal_16x4096", normal_bits(16, 4096, seed=7), prof)
        add(f"{prof}_tail_16x4096", heavy_tail_bits(16, 4096, seed=8), prof)
    add("sip_normal_4x12288", normal_bits(4, 12288, seed=9), "sip")
    # 32-weight blocks (the research block sizes the format admits)
    add("sip_tail_b32_7x100", heavy_tail_bits(7, 100, seed=5), "sip", block=32)
    add("gulp_tail_b32_7x100", heavy_tail_bits(7, 100, seed=5), "gulp", block=32)

    pins = {"packs": meta}
    # every bf16 pattern on a compressible background, every profile, blocks 32 / 1024
    ex = np.zeros((512, 513), np.uint16)
    ex.flat[:65536] = np.arange(65536, dtype=np.uint16)
    allpat = {}
    for prof in ("sip", "balanced", "gulp"):
        for block in (32, 1024):
            rpk = radix.pack_array(ex, compression_profile=prof, block_size=block)
            assert not rpk.raw and np.array_equal(radix.decode(rpk), ex)
            allpat[f"{prof}/{block}"] = {"sha256": sha(rpk.palette, rpk.offsets.astype(np.uint32),
                                                       rpk.data.astype(np.uint32)),
                                         "words": int(rpk.data.size), "palette": rpk.palette.tolist()}
    pins["all_patterns"] = allpat

    # config 1: 8B down_proj, seed 0, sip via the served packer; x seed 1
    g = torch.Generator().manual_seed(0)
    W = (torch.randn(4096, 12288, generator=g) * 0.02).to(torch.bfloat16)
    cfg = {}
    for prof in ("sip", "gulp"):
        p = pack_weight_served(W, compression_profile=prof)
        cfg[prof] = {"sha256": sha(p["rx_palette"], p["rx_offsets"], p["rx_data"]), "words": int(p["rx_data"].size),
                     "bpw": p["bpw"], "palette": p["rx_palette"].tolist(), "read_bytes": None}
        rt = to_device_radix(p, "cpu")
        cfg[prof]["read_bytes"] = int(radix_ops.read_bytes(rt))
        if prof == "sip":
            x = torch.randn(1, 12288, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
            mod = make_module(p, None, "cpu")
            y = mod(x)
            packs["config1/cpu_route_bf16"] = y.float().numpy()
            packs["config1/x_bf16"] = x.view(torch.int16).numpy().view(np.uint16)
    pins["config1"] = cfg
    np.savez_compressed(os.path.join(HERE, "packs.npz"), **packs)
    with open(os.path.join(HERE, "pins.json"), "w") as f:
        json.dump(pins, f, indent=1, sort_keys=True)
    print("wrote packs.npz and pins.json")


if __name__ == "__main__":
    main()
