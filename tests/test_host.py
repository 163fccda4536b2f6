"""Host logic with no GPU: the C ABI library loads and exports every entry
point the header declares; the loader's validation refuses malformed packs
with the reference's messages before touching the device; the launch
schedule, registry, pack reader and routing keep the reference's contract."""
from __future__ import annotations

import ctypes as ct
import os
import re

import numpy as np
import pytest

from conftest import ROOT, pack_of
from drinkme_b200 import _lib, codec, radix_schedule, registry


def test_library_exports_every_declared_entry_point():
    with open(os.path.join(ROOT, "include", "drinkme_b200.h")) as f:
        header = f.read()
    declared = set(re.findall(r"^int(?:64_t)? (dm_\w+)\(", header, flags=re.M))
    assert declared == set(_lib.EXPORTS)
    L = ct.CDLL(_lib.LIB_PATH)
    for name in declared:
        assert hasattr(L, name), name
    assert _lib.lib().dm_version() >= 100


def _create(p, row_begin=0, row_end=None):
    """dm_tensor_create up to its validation (no device is touched before it
    passes)."""
    pal = np.ascontiguousarray(p["rx_palette"], dtype=np.uint8)
    off = np.ascontiguousarray(p["rx_offsets"], dtype=np.uint32)
    data = np.ascontiguousarray(p["rx_data"], dtype=np.uint32)
    w = (ct.c_int32 * len(p["widths"]))(*[int(x) for x in p["widths"]])
    h = ct.c_void_p()
    R = int(p["R"])
    _lib.call("dm_tensor_create", pal.ctypes.data_as(ct.c_void_p), pal.size, off.ctypes.data_as(ct.c_void_p),
              off.size, data.ctypes.data_as(ct.c_void_p), data.size, R, int(p["C"]), w, len(p["widths"]),
              int(p["block_size"]), row_begin, R if row_end is None else row_end, 0, ct.byref(h))
    return h


def test_loader_refuses_malformed_descriptors(golden):
    z, pins = golden
    p = pack_of(z, pins, "sip_normal_16x4096")
    with pytest.raises(ValueError, match="invalid radix block offsets"):
        _create(dict(p, rx_offsets=p["rx_offsets"][:-1]))
    off = p["rx_offsets"].copy()
    off[1] = 1
    with pytest.raises(ValueError, match="fewer than the 352 its literal plane"):
        _create(dict(p, rx_offsets=off))
    with pytest.raises(ValueError, match="invalid radix palette entries"):
        _create(dict(p, rx_palette=np.zeros_like(p["rx_palette"])))
    with pytest.raises(ValueError, match="invalid radix block size"):
        _create(dict(p, block_size=1000))
    with pytest.raises(ValueError, match="2..8 widths"):
        _create(dict(p, widths=[3, 7]))


def test_fused_loader_refuses_parts_it_cannot_serve(golden):
    """dm_tensor_create_multi validates every part and the fusion rules on the
    host, before touching a device."""
    import torch

    from drinkme_b200.tensor import RadixTensor

    z, pins = golden
    p = pack_of(z, pins, "sip_normal_16x4096")
    g = torch.Generator().manual_seed(0)
    narrow = codec.pack_weight_radix((torch.randn(16, 2048, generator=g) * 0.02).to(torch.bfloat16), "sip")
    # ragged blocks: not re-encoded as sip, so never fusable
    gulp = codec.pack_weight_radix((torch.randn(16, 3079, generator=g) * 0.02).to(torch.bfloat16), "gulp")
    with pytest.raises(ValueError, match="invalid radix palette entries"):
        RadixTensor.fused([p, dict(p, rx_palette=np.zeros_like(p["rx_palette"]))], "cuda:0")
    with pytest.raises(ValueError, match="multiple of 16 rows"):
        RadixTensor.fused([p, p], "cuda:0", [(0, 13), (0, 16)])
    with pytest.raises(ValueError, match="share columns, block size and tier widths"):
        RadixTensor.fused([p, narrow], "cuda:0")
    with pytest.raises(ValueError, match="share columns, block size and tier widths"):
        RadixTensor.fused([p, gulp], "cuda:0")
    with pytest.raises(ValueError, match="served by the sip kernel"):
        RadixTensor.fused([gulp, gulp], "cuda:0")
    with pytest.raises(ValueError, match="one row range per pack"):
        RadixTensor.fused([p, p], "cuda:0", [(0, 16)])


def test_long_block_is_refused(golden):
    z, pins = golden
    p = pack_of(z, pins, "sip_normal_16x4096")
    off = p["rx_offsets"].astype(np.int64)
    data = np.insert(p["rx_data"], int(off[1]), np.zeros(400, np.uint32))
    off[1:] += 400
    with pytest.raises(ValueError, match="more than the 608 any block"):
        _create(dict(p, rx_offsets=off.astype(np.uint32), rx_data=data))


def test_codec_validate_tensor_messages(golden):
    z, pins = golden
    p = dict(pack_pack := pack_of(z, pins, "gulp_normal_16x4096"), format_version=1)
    codec.validate_tensor("a", p)
    with pytest.raises(ValueError, match=r"pack tensor a \(radix\): block_size"):
        codec.validate_tensor("a", dict(p, block_size=32))
    with pytest.raises(ValueError, match="at most four"):
        codec.validate_tensor("a", dict(p, widths=[2, 2, 2, 2, 8]))
    with pytest.raises(ValueError, match="1..4 bits"):
        codec.validate_tensor("a", dict(p, widths=[5, 8]))
    with pytest.raises(ValueError, match="profile"):
        codec.validate_tensor("a", dict(p, profile="nope"))
    with pytest.raises(ValueError, match="invalid radix palette entries"):
        codec.validate_tensor("a", dict(p, rx_palette=np.zeros_like(pack_pack["rx_palette"])))
    with pytest.raises(ValueError, match="codec"):
        codec.validate_tensor("a", dict(p, codec="fp8"))


def test_pack_dir_round_trip(tmp_path, golden):
    z, pins = golden
    tensors = {}
    for name in ("sip_normal_16x4096", "gulp_tail_16x4096"):
        p = pack_of(z, pins, name)
        tensors[name] = {**p, "bpw": float(p["bpw"])}
    tensors["raw"] = codec.raw_dict(np.zeros((4, 8), np.uint16))
    codec.save_pack_dir(str(tmp_path / "pk"), tensors, {"hfRepo": "x/y"})
    got = dict(codec.iter_pack_dir(str(tmp_path / "pk")))
    assert set(got) == set(tensors)
    for name in ("sip_normal_16x4096", "gulp_tail_16x4096"):
        for k in ("rx_palette", "rx_offsets", "rx_data"):
            assert np.array_equal(got[name][k], tensors[name][k])
    assert np.array_equal(got["raw"]["raw_bits"], tensors["raw"]["raw_bits"])


def test_pack_dir_refuses_other_versions_and_escaping_files(tmp_path, golden):
    import json

    z, pins = golden
    d = tmp_path / "pk"
    codec.save_pack_dir(str(d), {"a": pack_of(z, pins, "sip_normal_16x4096")}, {})
    meta = json.loads((d / "meta.json").read_text())
    (d / "meta.json").write_text(json.dumps(dict(meta, formatVersion=2)))
    with pytest.raises(ValueError, match="pack format 2"):
        list(codec.iter_pack_dir(str(d)))
    (d / "meta.json").write_text(json.dumps(dict(meta, tensors={"a": "../x.npz"})))
    with pytest.raises(ValueError, match="bare basename"):
        list(codec.iter_pack_dir(str(d)))


def test_schedule_shape_classes_and_overrides():
    assert radix_schedule.shape_class(151936, 4096) == "head"
    assert radix_schedule.shape_class(1024, 4096) == "narrow"
    assert radix_schedule.shape_class(4096, 12288) == "long"
    assert radix_schedule.shape_class(12288, 4096) == "wide"
    assert radix_schedule.shape_class(4096, 4096) == "square"
    assert radix_schedule.family((3, 8)) == "sip" and radix_schedule.family((2, 2, 4, 8)) == "scheduled"
    L = radix_schedule.select(4096, 4096, 1024, (3, 8))
    assert L.box_class == "b200" and L.kernel == "sip-mma-sm100a" and L.source == "table"
    assert L.knobs() == (0, 0, 4, 16)
    assert radix_schedule.select(4096, 4100, 1024, (3, 8)).kernel == "generic-sm100a"
    # gulp with whole 1024-weight blocks is re-encoded as sip by the loader
    assert radix_schedule.select(4096, 4096, 1024, (2, 2, 4, 8)).kernel == "sip-mma-sm100a"
    e = radix_schedule.select(4096, 4096, 1024, (3, 8), override="slots=3,split=tiles,skew=0,resident=0")
    assert e.knobs() == (3, 2, 0, 0) and e.source == "env"
    assert radix_schedule.select(1, 1, override="slots=rule").slots == 0
    assert radix_schedule.select(1, 1, override="spike").knobs() == (2, 2, 0, 0)
    for bad in ("slots=7", "split=rows", "skew=-1", "resident=17", "warps=4", "bogus=1"):
        with pytest.raises(ValueError):
            radix_schedule.select(1, 1, override=bad)
    per = radix_schedule.select(1024, 4096, override='{"narrow": {"slots": 2, "split": "stream"}}')
    assert per.knobs() == (2, 1, 4, 16)
    assert radix_schedule.select(4096, 4096, override='{"narrow": {"slots": 2}}').slots == 0  # other classes: the row
    with pytest.raises(ValueError):
        radix_schedule.select(1, 1, override='{"narrow": {"warps": 2}}')


def test_registry_rows():
    assert registry.supported("radix", 0, registry.GEMV, registry.CUDA_SM100)
    assert registry.supported("radix", 0, registry.MC, registry.CUDA_SM100)
    assert not registry.supported("radix", 0, registry.GEMV, registry.CPU)
    assert not registry.supported("fp8", 0, registry.GEMV, registry.CUDA_SM100)
    assert registry.kernel_of("cpu") == registry.CPU
    assert "unknown combination" in registry.unsupported_note("fp8", 0, registry.GEMV, registry.CUDA_SM100)


def test_routing_thresholds(monkeypatch):
    from drinkme_b200 import swap

    class Fake(swap.CompressedLinear):
        pass

    m = Fake({"R": 8, "C": 8, "codec": "radix"}, None)
    swap._DENSE_MIN = None
    monkeypatch.delenv("DRINKME_PREFILL_DENSE_MIN", raising=False)
    assert m._route_rows(1) == "gemv"
    assert [m._route_rows(k) for k in range(2, 9)] == ["mc"] * 7
    assert [m._route_rows(k) for k in range(9, 17)] == ["loop"] * 8  # the crossover measured on B200
    assert m._route_rows(17) == "dense" and swap.fused_m_max() == 8
    swap._DENSE_MIN = None
    monkeypatch.setenv("DRINKME_PREFILL_DENSE_MIN", "0")
    assert m._route_rows(9) == "loop" and m._route_rows(5) == "mc"
    swap._DENSE_MIN = None
    monkeypatch.setenv("DRINKME_PREFILL_DENSE_MIN", "4")
    assert m._route_rows(4) == "dense" and m._route_rows(3) == "mc"
    assert swap.fused_m_max() == 3  # an MTP verify batch stays below the dense arm
    swap._DENSE_MIN = None


def test_cpu_inputs_are_refused_not_served():
    import torch

    from drinkme_b200 import swap

    m = swap.CompressedLinear({"R": 8, "C": 8, "codec": "radix"}, None)
    with pytest.raises(ValueError, match="CUDA"):
        m(torch.zeros(1, 8))
    with pytest.raises(ValueError, match="CUDA"):
        swap.to_device_radix({"R": 1}, "cpu")


def test_stock_and_raw_gemv_modes(monkeypatch):
    """The reference's mode parsing (swap.py:665-781): an unknown mode is a
    ValueError naming the variable; off the accelerator the stock GEMV is
    F.linear and the raw GEMV "stock"; on it the defaults are this
    package's raw kernel ("b200") and "stock"."""
    from drinkme_b200 import swap

    monkeypatch.delenv(swap.STOCK_GEMV_ENV, raising=False)
    monkeypatch.delenv(swap.RAW_GEMV_ENV, raising=False)
    assert swap.stock_gemv_mode("cpu") == "linear"
    assert swap.stock_gemv_mode("cuda:0") == "b200"
    assert swap.raw_gemv_mode("cpu") == "stock" and swap.raw_gemv_mode("cuda:1") == "stock"
    monkeypatch.setenv(swap.STOCK_GEMV_ENV, "mv")
    assert swap.stock_gemv_mode("cuda:0") == "mv" and swap.stock_gemv_mode("cpu") == "linear"
    monkeypatch.setenv(swap.STOCK_GEMV_ENV, "fast")
    with pytest.raises(ValueError, match="DRINKME_STOCK_GEMV"):
        swap.stock_gemv_mode("cuda:0")
    monkeypatch.setenv(swap.RAW_GEMV_ENV, "twin")
    assert swap.raw_gemv_mode("cuda:0") == "twin"
    monkeypatch.setenv(swap.RAW_GEMV_ENV, "x")
    with pytest.raises(ValueError, match="DRINKME_RAW_GEMV"):
        swap.raw_gemv_mode("cuda:0")


def test_stock_linear_off_the_accelerator_is_f_linear():
    import torch

    from drinkme_b200 import swap

    g = torch.Generator().manual_seed(3)
    w = torch.randn(64, 1024, generator=g).to(torch.bfloat16)
    b = torch.randn(64, generator=g).to(torch.bfloat16)
    x = torch.randn(2, 1024, generator=g).to(torch.bfloat16)
    want = torch.nn.functional.linear(x, w, b)
    for mode in swap.STOCK_GEMV_MODES:
        assert torch.equal(swap.stock_linear(x, w, b, mode), want)
    assert torch.equal(swap.stock_linear(x, w, b, "b200", swap.raw_gemv_dict(64, 1024)), want)


def test_eligible_and_in_place_adoption():
    """Which Linears the codec takes (swap.py:850-854), and the raw routes'
    adoption: the Linear itself re-classed, its Parameters untouched; nothing
    is installed off the accelerator."""
    import torch

    from drinkme_b200 import swap

    big = torch.nn.Linear(1024, 2048, bias=False, dtype=torch.bfloat16)
    assert swap.eligible(big)
    assert not swap.eligible(torch.nn.Linear(1024, 64, dtype=torch.bfloat16))
    assert not swap.eligible(torch.nn.Linear(1024, 2048))  # fp32
    assert not swap.eligible(torch.nn.Linear(1026, 2048, dtype=torch.bfloat16))  # columns % 4
    assert not swap.eligible(torch.nn.Embedding(2048, 1024))
    w = big.weight
    got = swap.StockLinear.adopt(big, "mv")
    assert got is big and isinstance(big, swap.StockLinear) and big.weight is w and big.stock_gemv == "mv"
    m = torch.nn.Sequential(torch.nn.Linear(1024, 64, dtype=torch.bfloat16))
    assert not swap.codec_tree(m)
    assert swap.install_stock_gemv(m, "cpu", "b200") == 0
    assert swap.install_narrow(m, "cpu") == []


def test_chain_create_refuses_bad_arguments_without_a_gpu():
    """dm_chain_create checks its arguments before it touches a device: no
    links, M outside 1..8 (the reference's gemv_mc ValueError) and an output
    dtype other than bf16 / fp32 are refused with named errors."""
    import ctypes as ct

    arr = (_lib.ChainLink * 1)()
    out = ct.c_void_p()
    with pytest.raises(ValueError, match="no links"):
        _lib.call("dm_chain_create", arr, 0, 1, _lib.DM_BF16, ct.byref(out))
    with pytest.raises(ValueError, match="outside 1..8"):
        _lib.call("dm_chain_create", arr, 1, 9, _lib.DM_BF16, ct.byref(out))
    with pytest.raises(ValueError, match="dtype"):
        _lib.call("dm_chain_create", arr, 1, 1, 7, ct.byref(out))
    with pytest.raises(ValueError, match="null tensor"):
        _lib.call("dm_chain_create", arr, 1, 1, _lib.DM_BF16, ct.byref(out))
    with pytest.raises(ValueError, match="null chain"):
        _lib.call("dm_chain_run", None, None)
    assert ct.sizeof(_lib.ChainLink) == 224  # t, x, bias, dm_gather (192), wait: the header's layout
