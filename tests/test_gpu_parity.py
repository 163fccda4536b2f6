"""GPU parity: the sm_100a kernels, called through the C ABI, against the CPU
oracle (oracle/oracle.py) and against the reference's own outputs (the
golden vectors: its encoder's packs, its decoders' bits, its Triton kernels'
fp32 GEMVs).

Gates, as the reference states them:
  * decoded weights bit-exact (bench/radix_gemv_bitpin.py "bits");
  * GEMV within |y - y64| <= 2e-6 * |x|.|W| + 1e-7 of float64
    (bench/radix_gemv_bitpin.py:182, radix_mc_bitpin.py:104);
  * linear outputs within 1e-3 max relative error, max|y - y_ref| /
    max|y_ref|, of the reference's own kernels on the same inputs;
  * fused bias: the bf16 output == (fp32 + bias).to(bf16) exactly;
  * row m of an M-row call bitwise the M=1 call; bf16 x == its fp32
    widening (tests/test_narrow_linear.py:101-123).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import all_patterns, pack_of, radix_names
from drinkme_b200 import codec, radix_ops, swap
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _bits_t(U):
    return torch.from_numpy(np.ascontiguousarray(U).view(np.int16)).view(torch.bfloat16)


def _x_of(z, name, M=1):
    xb = z[f"{name}/x_bf16"][:M]
    return torch.from_numpy(xb.view(np.int16).copy()).view(torch.bfloat16).to(DEV)


def _f32(x):
    return x.float().cpu().numpy()


def _within_bound(y, x, bits):
    y64, bound = oracle.gemv_bound(_f32(x), bits)
    err = np.abs(y.astype(np.float64) - y64)
    return bool(np.all(err <= bound)), float((err / bound).max())


@pytest.fixture(scope="module")
def runtimes(golden):
    z, pins = golden
    out = {}
    for name in radix_names(pins):
        out[name] = swap.to_device_radix(pack_of(z, pins, name), DEV)
    return out


def test_decode_every_golden_pack_bit_exact(golden, runtimes):
    z, pins = golden
    for name, rt in runtimes.items():
        got = radix_ops.decode_bits(rt).cpu().numpy()
        assert np.array_equal(got.view(np.uint16), z[f"{name}/bits"]), name


@pytest.mark.parametrize("profile", ["sip", "balanced", "gulp"])
@pytest.mark.parametrize("block", [32, 1024])
def test_all_65536_patterns_decode_exactly(profile, block):
    ex = all_patterns()
    pal, off, data = codec.encode_arrays(ex, codec.PROFILES[profile], block)
    p = {"rx_palette": pal, "rx_offsets": off, "rx_data": data, "R": 512, "C": 513,
         "widths": list(codec.PROFILES[profile]), "block_size": block, "codec": "radix", "profile": profile}
    rt = swap.to_device_radix(p, DEV)
    got = radix_ops.decode_bits(rt).cpu().numpy().view(np.uint16)
    assert np.array_equal(got, ex)
    again = radix_ops.decode_bits(rt).cpu().numpy().view(np.uint16)
    assert np.array_equal(again, ex)


def test_gulp_schedule_matches_the_reference(golden, runtimes):
    z, pins = golden
    n = 0
    for name, rt in runtimes.items():
        key = f"{name}/schedule"
        if key in z.files:
            got = rt["rx_schedule"].cpu().numpy().view(np.uint16)
            assert np.array_equal(got, z[key]), name
            n += 1
    assert n >= 10


def test_gemv_m1_bf16_within_float64_bound_and_reference(golden, runtimes):
    z, pins = golden
    for name, rt in runtimes.items():
        bits = z[f"{name}/bits"]
        x = _x_of(z, name)
        y = radix_ops.gemv(rt, x[0]).cpu().numpy()
        ok, worst = _within_bound(y[None, :], x, bits)
        assert ok, (name, worst, radix_ops.decoder_of(rt))
        ref = z[f"{name}/gemv_bf16x"]
        rel = np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-30)
        assert rel <= 1e-3, (name, rel)


def test_fast_path_serves_the_sip_whole_block_tensors(runtimes):
    kinds = {name: radix_ops.decoder_of(rt) for name, rt in runtimes.items()}
    assert kinds["sip_normal_16x4096"] == radix_ops.DECODER_SIP_MMA
    assert kinds["sip_tail_16x4096"] == radix_ops.DECODER_SIP_MMA
    assert kinds["sip_normal_4x12288"] == radix_ops.DECODER_SIP_MMA
    # other profiles with whole 1024-weight blocks: re-encoded as sip by the loader
    assert kinds["gulp_normal_16x4096"] == radix_ops.DECODER_SIP_MMA
    assert kinds["balanced_normal_16x4096"] == radix_ops.DECODER_SIP_MMA
    # ragged blocks: the general kernel
    assert kinds["sip_tail_3x1025"] == radix_ops.DECODER_GENERIC
    assert kinds["gulp_tail_17x3079"] == radix_ops.DECODER_GENERIC
    assert kinds["gulp_tail_b32_7x100"] == radix_ops.DECODER_GENERIC


@pytest.mark.parametrize("profile", ["gulp", "balanced"])
def test_other_profiles_reencoded_as_sip_keep_their_bits_and_counts(profile):
    """A gulp / balanced pack served by the sip kernels: the loader decodes it
    and re-encodes it as sip; the bits stay the source's, the handle reports
    the pack's own widths, payload words and read_bytes, and the GEMV stays
    within the float64 bound for M = 1..8."""
    g = torch.Generator().manual_seed(21)
    W = (torch.randn(512, 8192, generator=g) * 0.02).to(torch.bfloat16)
    p = codec.pack_weight_radix(W, profile)
    rt = swap.to_device_radix(p, DEV)
    info = rt["rx_handle"].info
    assert radix_ops.decoder_of(rt) == radix_ops.DECODER_SIP_MMA
    assert tuple(info.widths[:info.nwidths]) == tuple(p["widths"])
    assert info.payload_words == p["rx_data"].size
    nb = 512 * 8
    pal_words = sum(((1 << w) - 1 + 3) // 4 for w in p["widths"][:-1])
    assert radix_ops.read_bytes(rt) == p["rx_data"].size * 4 + (nb + 1) * 4 + pal_words * 4 + (
        nb * 2 if len(p["widths"]) > 2 else 0)
    assert info.device_bytes_per_call > 0
    bits = codec.bits_of(W)
    assert np.array_equal(radix_ops.decode_bits(rt).cpu().numpy().view(np.uint16), bits)
    x = torch.randn(8, 8192, generator=g).to(torch.bfloat16).to(DEV)
    for M in (1, 2, 4, 8):
        ok, worst = _within_bound(radix_ops.gemv_mc(rt, x[:M]).cpu().numpy(), x[:M], bits)
        assert ok, (profile, M, worst)
    # a row shard re-encodes only its rows
    rs = swap.to_device_radix(p, DEV, 128, 320)
    assert np.array_equal(radix_ops.decode_bits(rs).cpu().numpy().view(np.uint16), bits[128:320])


def test_gemv_fp32_x_within_bound(golden, runtimes):
    z, pins = golden
    for name, rt in runtimes.items():
        x32 = torch.from_numpy(z[f"{name}/x_f32"]).to(DEV)
        y = radix_ops.gemv(rt, x32[0]).cpu().numpy()
        ok, worst = _within_bound(y[None, :], x32, z[f"{name}/bits"])
        assert ok, (name, worst)
        ref = z[f"{name}/gemv_f32x"]
        assert np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-30) <= 1e-3, name


def test_fused_bias_rounds_once(golden, runtimes):
    z, pins = golden
    for name, rt in runtimes.items():
        x = _x_of(z, name)
        bias = torch.from_numpy(z[f"{name}/bias_bf16"].view(np.int16).copy()).view(torch.bfloat16).to(DEV)
        y32 = radix_ops.gemv(rt, x[0])
        fused = radix_ops.gemv_fused(rt, x[0], bias, torch.bfloat16)
        assert torch.equal(fused[0], (y32 + bias.float()).to(torch.bfloat16)), name


def test_mc_rows_bitwise_the_m1_call_and_within_bound(golden, runtimes):
    z, pins = golden
    for name, rt in runtimes.items():
        x = _x_of(z, name, 8)
        ones = [radix_ops.gemv(rt, x[j]) for j in range(8)]
        for M in range(1, 9):
            ym = radix_ops.gemv_mc(rt, x[:M])
            for j in range(M):
                assert torch.equal(ym[j], ones[j]), (name, M, j)
        y8 = radix_ops.gemv_mc(rt, x).cpu().numpy()
        ok, worst = _within_bound(y8, x, z[f"{name}/bits"])
        assert ok, (name, worst)
        ref = z[f"{name}/mc8_bf16x"]
        assert np.abs(y8 - ref).max() / max(np.abs(ref).max(), 1e-30) <= 1e-3, name


@pytest.mark.parametrize("R,C", [(4096, 5120), (1024, 5120), (3000, 2048)])
def test_mc_rows_bitwise_the_m1_call_on_tensors_spanning_every_sm(R, C):
    """Tensors with units enough for several stream-K workers per SM: the
    work split must not change with M (nor with fp32 activations, whose
    split rows triple the staged activations)."""
    g = torch.Generator().manual_seed(R + C)
    W = (torch.randn(R, C, generator=g) * 0.02).to(torch.bfloat16)
    rt = swap.to_device_radix(codec.pack_weight_radix(W, "sip"), DEV)
    x = torch.randn(8, C, generator=g)
    for dt in (torch.bfloat16, torch.float32):
        xd = x.to(dt).to(DEV)
        ones = [radix_ops.gemv(rt, xd[j]) for j in range(8)]
        for M in (2, 3, 5, 8):
            ym = radix_ops.gemv_mc(rt, xd[:M])
            for j in range(M):
                assert torch.equal(ym[j], ones[j]), (dt, M, j)
    assert torch.equal(radix_ops.gemv_mc(rt, x[:4].to(torch.bfloat16).to(DEV)),
                       radix_ops.gemv_mc(rt, x[:4].to(torch.bfloat16).float().to(DEV)))


def test_escape_heavy_units_with_few_staging_slots():
    """Rows whose exponents spread far outside the seven tier-0 ones escape
    almost every weight: their 16-row units (~70 KB) leave room for only two
    or three staging slots, so a consumer group can reach a slot whose
    previous phase is still landing. Results stay exact and bitwise equal
    across M."""
    g = torch.Generator().manual_seed(77)
    R, C = 96, 8192
    W = torch.randn(R, C, generator=g) * 0.02
    e = torch.randint(-60, 60, (48, C), generator=g).float()
    sgn = torch.where(torch.rand(48, C, generator=g) < 0.5, -1.0, 1.0)
    W[16:64] = sgn * torch.exp2(e) * (1 + torch.rand(48, C, generator=g))
    W = W.to(torch.bfloat16)
    p = codec.pack_weight_radix(W, "sip")
    rt = swap.to_device_radix(p, DEV)
    assert radix_ops.decoder_of(rt) == radix_ops.DECODER_SIP_MMA
    bits = codec.bits_of(W)
    assert np.array_equal(radix_ops.decode_bits(rt).cpu().numpy().view(np.uint16), bits)
    x = (torch.randn(8, C, generator=g) * 2.0 ** -40).to(torch.bfloat16).to(DEV)
    ones = [radix_ops.gemv(rt, x[j]) for j in range(8)]
    for M in (1, 2, 3, 5, 8):
        ym = radix_ops.gemv_mc(rt, x[:M])
        for j in range(M):
            assert torch.equal(ym[j], ones[j]), (M, j)
        ok, worst = _within_bound(ym.cpu().numpy(), x[:M], bits)
        assert ok, (M, worst)


def test_bf16_x_equals_its_fp32_widening(golden, runtimes):
    z, pins = golden
    for name, rt in runtimes.items():
        x = _x_of(z, name, 3)
        assert torch.equal(radix_ops.gemv_mc(rt, x), radix_ops.gemv_mc(rt, x.float())), name


def test_mc_refuses_m_outside_one_to_eight(runtimes):
    rt = runtimes["sip_normal_16x4096"]
    for M in (0, 9):
        with pytest.raises(ValueError, match="outside 1"):
            radix_ops.gemv_mc(rt, torch.zeros(M, 4096, dtype=torch.bfloat16, device=DEV))


def test_the_bias_cancellation_keeps_its_residual():
    """tests/test_codec_bias_rounding.py: W columns 0, 1 = 1, x = (1, 1/256),
    bias -1: one rounding keeps 2^-8 on every arm and every profile."""
    R = C = 1024
    w = torch.zeros(R, C, dtype=torch.bfloat16)
    w[:, :2] = 1
    b = torch.full((R,), -1.0, device=DEV, dtype=torch.bfloat16)
    for prof in ("sip", "gulp"):
        pk = codec.pack_weight_radix(w, prof)
        assert pk["codec"] == "radix"
        mod = swap.make_module(pk, b, DEV)
        for n in (1, 3, 8, 9):
            x = torch.zeros(n, C, device=DEV, dtype=torch.bfloat16)
            x[:, 0] = 1
            x[:, 1] = 1 / 256
            y = mod(x)
            assert torch.all(y == 0.00390625), (prof, n)


def test_module_routes_match_the_arms(golden):
    z, pins = golden
    name = "sip_normal_16x4096"
    p = pack_of(z, pins, name)
    bias = torch.linspace(-0.1, 0.1, 16, device=DEV).to(torch.bfloat16)
    mod = swap.make_module(p, bias, DEV)
    W = _bits_t(z[f"{name}/bits"]).to(DEV)
    x = _x_of(z, name, 8)
    assert mod._route(x[:1]) == "gemv"
    assert torch.equal(mod(x[:1])[0], radix_ops.gemv_fused(mod.p, x[0], bias, torch.bfloat16)[0])
    assert mod._route(x[:5]) == "mc"
    y5 = mod(x[:5])
    assert torch.equal(y5, (radix_ops.gemv_mc(mod.p, x[:5]) + bias.float()).to(torch.bfloat16))
    xl = torch.randn(12, 4096, device=DEV).to(torch.bfloat16)
    assert mod._route(xl) == "loop"  # between MC_MAX and the measured dense threshold
    assert torch.equal(mod(xl), torch.cat([mod(xl[i:i + 1]) for i in range(12)]))
    xd = torch.randn(swap.DENSE_MIN_MEASURED, 4096, device=DEV).to(torch.bfloat16)
    assert mod._route(xd) == "dense"
    # the dense arm: the reference's own (exact decoded bits, then F.linear)
    assert torch.equal(mod(xd), torch.nn.functional.linear(xd, W, bias))
    # ... or, with DRINKME_B200_PREFILL=tc, the tensor-core prefill kernel
    old = swap._PREFILL_TC
    try:
        swap._PREFILL_TC = True
        yd = mod(xd)
    finally:
        swap._PREFILL_TC = old
    assert torch.equal(yd, radix_ops.prefill(mod.p, xd, bias, torch.bfloat16))
    # fp32 outputs within 1e-3 max relative error of F.linear in fp32
    ref = torch.nn.functional.linear(xd.float(), W.float())
    y32 = radix_ops.prefill(mod.p, xd, None, torch.float32)
    assert (y32 - ref).abs().max() / ref.abs().max() <= 1e-3
    assert torch.equal(yd, (y32 + bias.float()).to(torch.bfloat16))  # the bias in fp32, one rounding


@pytest.mark.parametrize("R", [13, 40, 1])
def test_ragged_tiles_on_the_fast_path(R):
    g = torch.Generator().manual_seed(R)
    W = (torch.randn(R, 4096, generator=g) * 0.02).to(torch.bfloat16)
    p = codec.pack_weight_radix(W, "sip")
    rt = swap.to_device_radix(p, DEV)
    assert radix_ops.decoder_of(rt) == radix_ops.DECODER_SIP_MMA
    bits = codec.bits_of(W)
    assert np.array_equal(radix_ops.decode_bits(rt).cpu().numpy().view(np.uint16), bits)
    x = torch.randn(8, 4096, generator=g).to(torch.bfloat16).to(DEV)
    for M in (1, 8):
        y = radix_ops.gemv_mc(rt, x[:M]).cpu().numpy()
        ok, worst = _within_bound(y, x[:M], bits)
        assert ok, (R, M, worst)


def test_row_shards_are_the_rows_of_the_whole():
    g = torch.Generator().manual_seed(5)
    R, C = 100, 8192
    W = (torch.randn(R, C, generator=g) * 0.02).to(torch.bfloat16)
    p = codec.pack_weight_radix(W, "sip")
    bits = codec.bits_of(W)
    x = torch.randn(2, C, generator=g).to(torch.bfloat16).to(DEV)
    for r0, r1 in ((0, 37), (37, 64), (64, 100), (0, 100)):
        rt = swap.to_device_radix(p, DEV, r0, r1)
        assert np.array_equal(radix_ops.decode_bits(rt).cpu().numpy().view(np.uint16), bits[r0:r1])
        y = radix_ops.gemv_mc(rt, x).cpu().numpy()
        ok, worst = _within_bound(y, x, bits[r0:r1])
        assert ok, (r0, r1, worst)


def test_config1_down_proj_full_size():
    """BASELINE configs[0] shapes on the GPU: 4096 x 12288 sip, seed 0, x seed 1:
    decode bit-exact, y within the float64 bound and 1e-3 of the reference's
    CPU route (bf16 output of F.linear over the decoded weight)."""
    import json
    import os

    from conftest import GOLDEN

    g = torch.Generator().manual_seed(0)
    W = (torch.randn(4096, 12288, generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn(1, 12288, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    p = codec.pack_weight_served(W)
    rt = swap.to_device_radix(p, DEV)
    bits = codec.bits_of(W)
    assert np.array_equal(radix_ops.decode_bits(rt).cpu().numpy().view(np.uint16), bits)
    xd = x.to(DEV)
    y = radix_ops.gemv(rt, xd[0]).cpu().numpy()
    ok, worst = _within_bound(y[None, :], xd, bits)
    assert ok, worst
    z = np.load(os.path.join(GOLDEN, "packs.npz"))
    ref = z["config1/cpu_route_bf16"][0]
    yb = radix_ops.gemv_fused(rt, xd[0], None, torch.bfloat16).float().cpu().numpy()[0]
    assert np.abs(yb - ref).max() / np.abs(ref).max() <= 1e-2  # both bf16-rounded
    assert np.abs(y - ref).max() / np.abs(ref).max() <= 5e-3
    with open(os.path.join(GOLDEN, "pins.json")) as f:
        assert radix_ops.read_bytes(rt) == json.load(f)["config1"]["sip"]["read_bytes"]
    # the reference's own arithmetic at full size with fp32 outputs: its
    # native decoder's weight (oracle/_ref, bit-exact to the source) and an
    # fp32-accumulated product, the contract of its GEMV (radix_kernel_gpu.py:
    # 683-718); north_star's bar is 1e-3 max relative error
    if oracle.reference_native() is not None:
        Wref = oracle.reference_decode(p)
        assert np.array_equal(Wref, bits)
        Wf = torch.from_numpy(Wref.view(np.int16).copy()).view(torch.bfloat16).to(DEV).float()
        y32 = (xd.float() @ Wf.T)[0].cpu().numpy()
        rel = np.abs(y - y32).max() / np.abs(y32).max()
        assert rel <= 1e-3, rel


@pytest.mark.parametrize("shape", [(48, 5120), (32, 4096), (256, 6656)])
def test_raw_narrow_gemv(shape):
    R, C = shape
    torch.manual_seed(2)
    w = (torch.randn(R, C) * 0.05).to(torch.bfloat16).to(DEV)
    bias = (torch.randn(R) * 0.5).to(torch.bfloat16).to(DEV)
    x = (torch.randn(8, C, device=DEV) * 0.5).to(torch.bfloat16)
    ones = [radix_ops.gemv_narrow(w, x[j:j + 1], bias) for j in range(8)]
    for M in range(1, 9):
        ym = radix_ops.gemv_narrow(w, x[:M], bias)
        for j in range(M):
            assert torch.equal(ym[j:j + 1], ones[j]), (shape, M, j)
    y32 = radix_ops.gemv_raw(w, x, None, torch.float32).cpu().numpy()
    bits = w.cpu().view(torch.int16).numpy().view(np.uint16)
    y64, bound = oracle.gemv_bound(_f32(x), bits)
    assert np.all(np.abs(y32 - y64) <= bound)
    assert torch.equal(radix_ops.gemv_narrow(w, x[:3], None).float(),
                       radix_ops.gemv_narrow(w, x[:3].float(), None).to(torch.bfloat16).float())


def test_raw_gemv_adds_the_bias_before_the_one_rounding():
    lin = torch.zeros(2, 1024, dtype=torch.bfloat16, device=DEV)
    lin[0, 0] = 1.0
    lin[0, 1] = 1.0
    bias = torch.zeros(2, dtype=torch.bfloat16, device=DEV)
    bias[0] = -1.0
    x = torch.zeros(1, 1024, dtype=torch.bfloat16, device=DEV)
    x[0, 0] = 1.0
    x[0, 1] = 2.0 ** -9
    assert radix_ops.gemv_narrow(lin, x, bias)[0, 0].item() == 2.0 ** -9


def test_prepare_schedule_on_the_original_layout(golden):
    z, pins = golden
    name = "gulp_tail_16x4096"
    p = pack_of(z, pins, name)
    data = torch.from_numpy(p["rx_data"].view(np.int32).copy()).to(DEV)
    off = torch.from_numpy(p["rx_offsets"].view(np.int32).copy()).to(DEV)
    s = radix_ops.prepare_schedule(data, off, p["C"], p["widths"], 1024, 16 * 4)
    assert np.array_equal(s.cpu().numpy().view(np.uint16), z[f"{name}/schedule"])


def test_repeated_calls_are_bitwise_deterministic(runtimes, golden):
    z, _ = golden
    for name in ("sip_normal_16x4096", "sip_normal_4x12288", "gulp_normal_16x4096"):
        rt = runtimes[name]
        x = _x_of(z, name, 4)
        a = radix_ops.gemv_mc(rt, x)
        for _ in range(3):
            assert torch.equal(radix_ops.gemv_mc(rt, x), a)


def test_no_device_errors_recorded(runtimes):
    for name, rt in runtimes.items():
        assert rt["rx_handle"].device_error() == 0, name


def test_stock_linear_modes_on_the_gpu(monkeypatch):
    """The raw Linears' one-row routes (swap.py:681-742): "b200" / "triton"
    and a raw descriptor run the raw GEMV (fp32 accumulate, bias, one
    rounding: bitwise dm_gemv_raw), "mv" torch.mv / addmv, "linear"
    F.linear; all within bf16 rounding of a float64 reference, and M = 9
    always F.linear. StockLinear adopts a Linear in place, without a copy."""
    g = torch.Generator().manual_seed(9)
    w = (torch.randn(2048, 1024, generator=g) * 0.02).to(torch.bfloat16).to(DEV)
    b = (torch.randn(2048, generator=g) * 0.1).to(torch.bfloat16).to(DEV)
    x = torch.randn(1, 1024, generator=g).to(torch.bfloat16).to(DEV)
    ref = (x.double() @ w.double().t() + b.double()).float()
    raw = radix_ops.gemv_raw(w, x, b, torch.bfloat16)
    for mode, r in (("b200", None), ("triton", None), ("linear", swap.raw_gemv_dict(2048, 1024))):
        assert torch.equal(swap.stock_linear(x, w, b, mode, r), raw), mode
    for mode in ("mv", "linear"):
        y = swap.stock_linear(x, w, b, mode)
        assert y.shape == (1, 2048) and y.dtype == torch.bfloat16
        assert torch.allclose(y.float(), ref, rtol=2 ** -7, atol=1e-3), mode
    x9 = torch.randn(9, 1024, generator=g).to(torch.bfloat16).to(DEV)
    assert torch.equal(swap.stock_linear(x9, w, b, "b200"), torch.nn.functional.linear(x9, w, b))
    lin = torch.nn.Linear(1024, 2048, device=DEV, dtype=torch.bfloat16)
    model = torch.nn.Sequential(lin)
    assert swap.install_stock_gemv(model, DEV, "b200") == 1
    assert model[0] is lin and isinstance(lin, swap.StockLinear)
    assert torch.equal(model[0](x), swap.stock_linear(x, lin.weight, lin.bias, "b200"))


def test_runtime_dict_carries_the_reference_device_arrays():
    """to_device_radix's dict has the reference's device keys (swap.py:80-161)
    that reference code reads: rx_data's device (radix_ops.py:426, swap.py:
    433), rx_offsets / rx_palette / rx_schedule for read_bytes' formula
    (radix_ops.py:435-441), which must give this package's count."""
    g = torch.Generator().manual_seed(41)
    for R, C, prof, rows in ((300, 4096, "gulp", (0, 300)), (4096, 12288, "sip", (1024, 2048)),
                             (40, 1000, "sip", (0, 40))):
        W = (torch.randn(R, C, generator=g) * 0.02).to(torch.bfloat16)
        p = codec.pack_weight_radix(W, prof)
        rt = swap.to_device_radix(p, DEV, *rows)
        for k in ("rx_data", "rx_offsets", "rx_palette", "rx_schedule"):
            assert rt[k].device == torch.device(DEV), k
        nb = -(-C // 1024)
        assert rt["rx_offsets"].numel() == (rows[1] - rows[0]) * nb + 1
        off = np.asarray(p["rx_offsets"], dtype=np.int64)[rows[0] * nb:rows[1] * nb + 1]
        assert np.array_equal(rt["rx_offsets"].cpu().view(torch.int32).numpy().astype(np.int64), off - off[0])
        assert np.array_equal(rt["rx_palette"].cpu().view(torch.int32).numpy().view(np.uint32),
                              codec.padded_palette_words(p))
        formula = int(rt["NW"]) * 4 + sum(rt[k].numel() * rt[k].element_size()
                                          for k in ("rx_offsets", "rx_palette", "rx_schedule"))
        assert formula == radix_ops.read_bytes(rt)
        assert rt["rx_data"].numel() * 4 == rt["rx_handle"].info.layout_bytes
        assert swap.resident_bytes(rt) >= rt["rx_handle"].info.resident_bytes


def test_config3_gulp_full_size_rows():
    """BASELINE configs[2] at full size: the Qwen3-8B gate shape (12288 x
    4096) packed gulp, M = 2, 4 and 8 activation rows seeded per row: fp32
    outputs within 1e-3 max relative error of an fp32-accumulated product
    with the decoded (bit-exact) weight, and every row bitwise the M = 1
    call's."""
    g = torch.Generator().manual_seed(12)
    W = (torch.randn(12288, 4096, generator=g) * 0.02).to(torch.bfloat16)
    p = codec.pack_weight_radix(W, "gulp")
    assert p["codec"] == "radix" and p["profile"] == "gulp"
    rt = swap.to_device_radix(p, DEV)
    Wf = W.to(DEV).float()
    x = torch.cat([torch.randn(1, 4096, generator=torch.Generator().manual_seed(100 + m)) for m in range(8)])
    xd = x.to(torch.bfloat16).to(DEV)
    ones = [radix_ops.gemv_mc(rt, xd[m:m + 1]) for m in range(8)]
    for M in (2, 4, 8):
        y = radix_ops.gemv_mc(rt, xd[:M])
        ref = xd[:M].float() @ Wf.T
        assert (y - ref).abs().max() / ref.abs().max() <= 1e-3, M
        for m in range(M):
            assert torch.equal(y[m:m + 1], ones[m]), (M, m)
