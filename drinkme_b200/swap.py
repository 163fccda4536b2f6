"""The operator boundary: packed Linears served by the sm_100a kernels — the
drop-in for the reference's ``drinkme.codec.swap`` module classes and loader
(src/drinkme/codec/swap.py):

  to_device_radix(pack, device)   swap.py:80-161   the loader (here: the C
                                                   library's unit-major B200
                                                   layout, optionally one row
                                                   shard of the tensor)
  to_device_raw(pack, device)     swap.py:64-77
  CompressedLinear                swap.py:228-392  routing by M, epilogue
  RadixCompressedLinear           swap.py:395-456
  RawLinear                       swap.py:459-497
  NarrowLinear, install_narrow    swap.py:530-626
  stock_linear, StockLinear,      swap.py:660-849  the raw bf16 Linears'
  stock_gemv_mode, raw_gemv_mode,                  one-row GEMV choice
  install_stock_gemv, codec_tree
  make_module(pack, bias, device) swap.py:900-919
  eligible                        swap.py:850-854  which Linears the codec takes

Routing (swap.py:302-335): M == 1 -> "gemv"; 2 <= M <= MC_MAX -> "mc"
unless DRINKME_PREFILL_DENSE_MIN says dense; M >= the dense threshold ->
"dense" (decode the weight once, then one GEMM); "loop" in between and when
the dense arm is switched off, here through the multi-column kernel in
chunks of MC_MAX rows (same bits as one row at a time). The threshold is
DRINKME_PREFILL_DENSE_MIN when set, else the crossover measured on B200
(DENSE_MIN_MEASURED = 17; the reference's box measured GEMM_MIN_ROWS = 9). The epilogue rounds once: fp32 accumulate, plus the bias
in fp32, one cast (swap.py:284-300). There is no CPU route: a CPU input
raises (the reference's CPU route is the oracle here, oracle/oracle.py).
"""
from __future__ import annotations

import os
import warnings

import numpy as np
import torch

from . import codec, radix_ops
from .ops import MC_MAX
from .radix_schedule import select as select_launch
from .tensor import RadixTensor, device_view


def _cuda_device(device) -> torch.device:
    dev = torch.device(device)
    if dev.type != "cuda":
        raise ValueError(f"drinkme_b200 serves CUDA devices only, not {dev} (no CPU route)")
    return dev


def to_device_raw(pack: dict, device="cuda") -> dict:
    dev = _cuda_device(device)
    R, C = int(pack["R"]), int(pack["C"])
    bits = np.ascontiguousarray(pack["raw_bits"], dtype=np.uint16).reshape(R, C)
    w = torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16).to(dev)
    return {"weight": w, "R": R, "C": C, "codec": "raw", "format_version": codec.FORMAT_VERSION, "layout": 0}


def to_device_radix(pack: dict, device="cuda", row_begin: int = 0, row_end: int | None = None) -> dict:
    """A radix tensor dict -> its runtime dict on a CUDA device, rows
    [row_begin, row_end) of it (the whole tensor by default). The payload is
    validated and laid out by the C library; the gulp schedule is computed
    on the device over the pack's original layout (radix_ops.prepare_schedule)."""
    dev = _cuda_device(device)
    R, C = int(pack["R"]), int(pack["C"])
    widths = tuple(int(w) for w in pack["widths"])
    B = int(pack["block_size"])
    r0, r1 = int(row_begin), R if row_end is None else int(row_end)
    h = RadixTensor(pack, dev, r0, r1)
    launch = select_launch(R, C, B, widths)
    if h.info.fast_path:
        h.set_launch(*launch.knobs())
    nb = (C + B - 1) // B
    rows = r1 - r0
    if len(widths) > 2:
        off = np.ascontiguousarray(pack["rx_offsets"], dtype=np.uint32)[r0 * nb:r1 * nb + 1].astype(np.int64)
        data = np.ascontiguousarray(pack["rx_data"], dtype=np.uint32)[int(off[0]):int(off[-1])]
        d_data = torch.from_numpy(data.view(np.int32).copy()).to(dev)
        d_off = torch.from_numpy((off - off[0]).astype(np.int32)).to(dev)
        schedule = radix_ops.prepare_schedule(d_data, d_off, C, widths, B, rows * nb)
        del d_data, d_off
    else:
        schedule = torch.empty(0, dtype=torch.uint16, device=dev)
    pad = int(codec.block_word_bounds(B, codec.MANT, codec.EXP, widths)[1])
    # the reference's device arrays (swap.py:80-161), for callers that read
    # the dict: the shard's word directory (rebased) and the padded palette
    # words, verbatim; rx_data is the device payload the kernels stream, in
    # this package's B200 layout (unit-major, code planes), not pack order —
    # its .device and size are what reference code reads (radix_ops.py:426,
    # swap.py:433); NW and read_bytes stay the pack's
    off = np.ascontiguousarray(pack["rx_offsets"], dtype=np.uint32)[r0 * nb:r1 * nb + 1].astype(np.int64)
    d_offsets = torch.from_numpy((off - off[0]).astype(np.uint32)).to(dev)
    d_palette = torch.from_numpy(codec.padded_palette_words(pack)).to(dev)
    d_data = device_view(h.info.layout_ptr, (h.info.layout_bytes // 4,), torch.int32, dev).view(torch.uint32)
    return {
        **{k: v for k, v in pack.items() if k not in ("rx_palette", "rx_offsets", "rx_data")},
        "rx_handle": h,
        "rx_data": d_data, "rx_offsets": d_offsets, "rx_palette": d_palette, "rx_layout": "b200-unit-major",
        "rx_schedule": schedule,
        "rx_palette_np": np.ascontiguousarray(pack["rx_palette"], dtype=np.uint8),
        "rx_launch": launch.as_dict(),
        "NW": int(h.info.payload_words), "rx_pad_words": pad,
        "R": rows, "C": C, "R_full": R, "row_begin": r0, "widths": widths, "block_size": B, "NBK": rows * nb,
        "codec": "radix", "format_version": codec.FORMAT_VERSION, "layout": 0,
    }


def to_device_radix_fused(packs, device="cuda", ranges=None) -> dict:
    """Several sip radix tensors reading the same activations (q, k, v;
    gate, up) -> ONE runtime dict whose GEMV computes their outputs side by
    side, [M, sum of rows] (dm_tensor_create_multi). `ranges` optionally
    gives each pack's (row_begin, row_end) — a rank's row shard of each.
    The dict serves every radix_ops GEMV arm; `split_fused` cuts an output
    into the parts' views. No reference counterpart: the reference runs one
    RadixCompressedLinear per projection (swap.py:395-456)."""
    dev = _cuda_device(device)
    packs = list(packs)
    if not packs:
        raise ValueError("to_device_radix_fused: no tensors")
    ranges = [(int(a), int(pk["R"]) if b is None else int(b))
              for pk, (a, b) in zip(packs, ranges or [(0, None)] * len(packs))]
    h = RadixTensor.fused(packs, dev, ranges)
    C = int(packs[0]["C"])
    B = int(packs[0]["block_size"])
    widths = tuple(int(w) for w in packs[0]["widths"])
    rows = int(h.info.rows)
    launch = select_launch(rows, C, B, widths)
    h.set_launch(*launch.knobs())
    return {
        "rx_handle": h,
        "rx_schedule": torch.empty(0, dtype=torch.uint16, device=dev),
        "rx_launch": launch.as_dict(),
        "NW": int(h.info.payload_words),
        "R": rows, "C": C, "R_full": rows, "row_begin": 0, "widths": widths, "block_size": B,
        "NBK": int(h.info.nblocks), "codec": "radix", "format_version": codec.FORMAT_VERSION, "layout": 0,
        "fused_rows": tuple(b - a for a, b in ranges),
    }


def split_fused(runtime: dict, y: torch.Tensor):
    """The parts' outputs of a fused GEMV result [M, sum of rows], as views."""
    return torch.split(y, list(runtime["fused_rows"]), dim=-1)


def resident_bytes(runtime: dict) -> int:
    """Device bytes a runtime dict holds (pack.resident_bytes, pack.py:1170);
    rx_data, a view of the handle's own layout, is counted with the handle."""
    n = sum(v.numel() * v.element_size() for k, v in runtime.items()
            if torch.is_tensor(v) and not (k == "rx_data" and "rx_layout" in runtime))
    h = runtime.get("rx_handle")
    return n + (int(h.info.resident_bytes) if h is not None else 0)


_DENSE_MIN: int | None = None

# The dense arm's row threshold measured on B200 (bench.crossover_8b, one
# Qwen3-8B layer of sip linears): the row loop through the multi-column
# kernel, MC_MAX rows per launch, takes 208-228 us per layer at 9-16 rows
# (two launches per linear) against 275-277 us for decode + cuBLAS, and 336
# us at 24 rows (three) — so the dense arm starts at 17 rows here, where the
# reference box measured GEMM_MIN_ROWS = 9.
DENSE_MIN_MEASURED = 2 * MC_MAX + 1


def _dense_min() -> int:
    """DRINKME_PREFILL_DENSE_MIN if set, else the measured crossover; <= 0
    disables the dense arm. Read once (swap.py:205-225)."""
    global _DENSE_MIN
    if _DENSE_MIN is None:
        raw = os.environ.get("DRINKME_PREFILL_DENSE_MIN", "").strip()
        try:
            _DENSE_MIN = int(raw) if raw else DENSE_MIN_MEASURED
        except ValueError:
            warnings.warn(f"DRINKME_PREFILL_DENSE_MIN={raw!r} is not an integer; using the measured default "
                          f"{DENSE_MIN_MEASURED}")
            _DENSE_MIN = DENSE_MIN_MEASURED
    return _DENSE_MIN


_PREFILL_TC: bool | None = None


def _prefill_kernel() -> bool:
    """DRINKME_B200_PREFILL=tc routes the dense arm of sip tensors through the
    tensor-core prefill kernel (radix_ops.prefill); by default the dense arm
    is the reference's own (decode to bf16, then one cuBLAS GEMM), which
    measures faster on B200 today. Read once."""
    global _PREFILL_TC
    if _PREFILL_TC is None:
        _PREFILL_TC = os.environ.get("DRINKME_B200_PREFILL", "").strip().lower() == "tc"
    return _PREFILL_TC


class CompressedLinear(torch.nn.Module):
    """Routing by M and the round-once epilogue, shared by the radix and raw
    modules."""

    GEMM_MIN_ROWS = MC_MAX + 1

    def __init__(self, runtime: dict, bias):
        super().__init__()
        self.p = runtime
        self.bias = bias
        self.R, self.C = int(runtime["R"]), int(runtime["C"])
        self.tensor_codec = runtime.get("codec")
        self.layout = int(runtime.get("layout", 0))

    def _gemv_row(self, xi):
        raise NotImplementedError

    def _gemv_cols(self, xm):
        raise NotImplementedError

    def _dense_weight(self):
        raise NotImplementedError

    def _epilogue(self, y, x, shape):
        if self.bias is not None:
            y = y + self.bias
        return y.to(x.dtype).reshape(*shape[:-1], self.R)

    def _route(self, x) -> str:
        if x.device.type != "cuda":
            raise ValueError(f"drinkme_b200 serves CUDA tensors only; got an input on {x.device} "
                             "(the CPU reference route is not part of this package)")
        return self._route_rows(x.numel() // x.shape[-1])

    def _route_rows(self, m: int) -> str:
        if m == 1:
            return "gemv"
        dense_min = _dense_min()
        if 0 < dense_min <= m:
            return "dense"
        if m <= MC_MAX:
            return "mc"
        return "loop"

    def forward(self, x):
        return self._forward(x, self._route(x))

    def _forward(self, x, route: str):
        shape = x.shape
        xf = x.reshape(-1, self.C)
        if route == "gemv":
            return self._epilogue(self._gemv_row(xf[0].float().contiguous()), x, shape)
        if route == "dense":
            W = self._dense_weight()
            out = torch.nn.functional.linear(xf, W, self.bias).reshape(*shape[:-1], self.R)
            del W
            return out
        if route == "mc":
            return self._epilogue(self._gemv_cols(xf.float().contiguous()), x, shape)
        outs = torch.empty(xf.shape[0], self.R, device=x.device, dtype=torch.float32)
        for i in range(xf.shape[0]):
            outs[i] = self._gemv_row(xf[i].float().contiguous())
        return self._epilogue(outs, x, shape)


class RadixCompressedLinear(CompressedLinear):
    """A radix-coded Linear served by the fused decode + GEMV kernels: the
    gemv and mc routes read x in its own dtype (bf16 or fp32) and fuse the
    bias and the one rounding in the kernel."""

    def __init__(self, runtime: dict, bias):
        if runtime.get("codec") != "radix" or "rx_handle" not in runtime:
            raise ValueError("RadixCompressedLinear needs a to_device_radix runtime dict")
        super().__init__(runtime, bias)
        self.tensor_codec = "radix"

    def _gemv_row(self, xi):
        return radix_ops.gemv(self.p, xi)

    def _gemv_cols(self, xm):
        return radix_ops.gemv_mc(self.p, xm)

    def _dense_weight(self):
        return radix_ops.decode_weight(self.p)

    def _forward(self, x, route: str):
        if route in ("gemv", "mc") and x.dtype in (torch.bfloat16, torch.float32):
            shape = x.shape
            xf = x.reshape(-1, self.C)
            if route == "gemv":
                out = radix_ops.gemv_fused(self.p, xf[0], self.bias, x.dtype)
            else:
                out = radix_ops.gemv_mc_fused(self.p, xf, self.bias, x.dtype)
            return out.reshape(*shape[:-1], self.R)
        if route == "loop" and x.dtype in (torch.bfloat16, torch.float32):
            return self._loop_rows(x, x.shape)
        if route == "dense" and x.dtype == torch.bfloat16 and _prefill_kernel() and self.p["rx_handle"].info.fast_path:
            # the dense arm's arithmetic on the tensor cores, the weights
            # decoded into shared memory instead of HBM
            shape = x.shape
            out = radix_ops.prefill(self.p, x.reshape(-1, self.C), self.bias, x.dtype)
            return out.reshape(*shape[:-1], self.R)
        return super()._forward(x, route)


    def _loop_rows(self, x, shape):
        # the row loop in chunks of MC_MAX rows through the multi-column
        # kernel: each row bitwise the M = 1 call (the reference loops one
        # row at a time, swap.py:380-392), the weight read once per chunk
        xf = x.reshape(-1, self.C)
        out = torch.empty(xf.shape[0], self.R, device=x.device, dtype=x.dtype)
        for i in range(0, xf.shape[0], MC_MAX):
            radix_ops.gemv_into(self.p, xf[i:i + MC_MAX], self.bias, out[i:i + MC_MAX])
        return out.reshape(*shape[:-1], self.R)


def fused_m_max() -> int:
    """The widest MTP verify batch whose compressed Linears stay on the serial
    step's numerics (serving/mtp.py:228-240 FUSED_M_MAX): the multi-column
    kernel serves 2..MC_MAX rows, each bitwise the M = 1 answer, up to the
    row before the dense arm takes over."""
    dense_min = _dense_min()
    return MC_MAX if dense_min <= 0 else max(1, min(MC_MAX, dense_min - 1))


class RawLinear(CompressedLinear):
    """The raw fallback (bf16 bits verbatim): stock_linear under the module's
    stock GEMV mode — by default this package's raw GEMV for 1..MC_MAX rows,
    cuBLAS (F.linear) above."""

    stock_gemv = "b200"
    raw_gemv = None  # raw_gemv_dict's dict once install_stock_gemv has given one

    def __init__(self, runtime: dict, bias):
        if runtime.get("codec") != "raw":
            raise ValueError("RawLinear needs a to_device_raw runtime dict")
        super().__init__(runtime, bias)
        self.tensor_codec = "raw"

    def _dense_weight(self):
        return self.p["weight"]

    def forward(self, x):
        self._route(x)
        return stock_linear(x, self.p["weight"], self.bias, self.stock_gemv, self.raw_gemv)


# The stock GEMV of a raw bf16 Linear's small-M call (swap.py:660-708): the
# reference picks it per AMD gfx target ("linear", "mv", "triton"; "linear"
# elsewhere). On B200 the default is "b200", this package's raw GEMV (the
# Qwen3-8B lm_head, 151936 x 4096, one row: 180.8 us against cuBLAS's
# 203.1 us); "triton", the reference's twin kernel, maps to the same kernel.
# DRINKME_STOCK_GEMV overrides, with the reference's name and check.
STOCK_GEMV_ENV = "DRINKME_STOCK_GEMV"
STOCK_GEMV_MODES = ("linear", "mv", "triton", "b200")
RAW_GEMV_ENV = "DRINKME_RAW_GEMV"
RAW_GEMV_MODES = ("stock", "twin")


def stock_gemv_mode(device) -> str:
    """DRINKME_STOCK_GEMV when set to a mode, else "b200"; always "linear"
    off the accelerator (swap.py:665-679)."""
    spec = os.environ.get(STOCK_GEMV_ENV, "auto").strip() or "auto"
    if spec not in ("auto",) + STOCK_GEMV_MODES:
        raise ValueError(f"{STOCK_GEMV_ENV}={spec!r}: one of auto, {', '.join(STOCK_GEMV_MODES)}")
    if not str(device).startswith("cuda"):
        return "linear"
    return "b200" if spec == "auto" else spec


def raw_gemv_mode(device) -> str:
    """DRINKME_RAW_GEMV when set to a mode, else "stock"; always "stock" off
    the accelerator (swap.py:768-781). "twin" sends a codec tree's raw
    Linears through this package's raw GEMV whatever the stock mode."""
    spec = os.environ.get(RAW_GEMV_ENV, "auto").strip() or "auto"
    if spec not in ("auto",) + RAW_GEMV_MODES:
        raise ValueError(f"{RAW_GEMV_ENV}={spec!r}: one of auto, {', '.join(RAW_GEMV_MODES)}")
    if not str(device).startswith("cuda"):
        return "stock"
    return "stock" if spec == "auto" else spec


def codec_tree(model) -> bool:
    """Does the tree hold a codec module (swap.py:784-789)?"""
    return any(isinstance(m, CompressedLinear) for m in model.modules())


def raw_gemv_dict(R: int, C: int) -> dict:
    """The descriptor a raw [R, C] Linear's small-M call runs the raw GEMV
    under (swap.py:792-803: the reference's twin-kernel launch row; this
    kernel needs no schedule, so only the shape and the kernel's name)."""
    return {"R": int(R), "C": int(C), "codec": "raw", "kernel": "gemv_raw_sm100a"}


def stock_linear(x, weight, bias, mode: str = "b200", raw: dict | None = None):
    """A raw bf16 Linear's forward under the stock GEMV `mode`
    (swap.py:681-707): "b200" / "triton", or any `raw` descriptor, sends
    1..MC_MAX rows on the accelerator through the raw GEMV (fp32 accumulate,
    the bias added in fp32, one rounding); "mv" sends one row through
    torch.mv (torch.addmv with a bias) with cuBLASLt preferred for the call;
    everything else is F.linear."""
    M = x.numel() // x.shape[-1] if x.numel() else 0
    kernel = raw is not None or mode in ("b200", "triton")
    if (kernel and x.device.type == "cuda" and 1 <= M <= MC_MAX and weight.dtype == torch.bfloat16
            and x.dtype in (torch.bfloat16, torch.float32) and weight.is_contiguous()):
        y = radix_ops.gemv_raw(weight, x.reshape(M, -1), bias, x.dtype)
        return y.reshape(*x.shape[:-1], weight.shape[0])
    if mode == "mv" and x.device.type == "cuda" and x.numel() == weight.shape[1]:
        # one row as a matrix-vector product on the default BLAS backend (the
        # reference's "mv" prefers hipBLASLt for its AMD targets; on B200
        # cuBLAS chooses its own GEMV kernel)
        v = x.reshape(weight.shape[1])
        y = weight.mv(v) if bias is None else bias.addmv(weight, v)
        return y.reshape(*x.shape[:-1], weight.shape[0])
    return torch.nn.functional.linear(x, weight, bias)


def _raw_bf16_linear(mod, min_rows: int, max_rows: int | None, min_cols: int) -> bool:
    """A plain torch Linear with a bf16 CUDA weight of the given extents."""
    if type(mod) is not torch.nn.Linear:
        return False
    w = mod.weight
    if w.dtype != torch.bfloat16 or w.device.type != "cuda":
        return False
    rows, cols = w.shape
    return rows >= min_rows and cols >= min_cols and (max_rows is None or rows <= max_rows)


class StockLinear(torch.nn.Linear):
    """A raw bf16 Linear with both dims >= 1024 (a tied lm_head, the stock
    arm's Linears) whose forward is stock_linear's (swap.py:710-742): the
    checkpoint's own Parameters, adopted without a copy."""

    stock_gemv = "b200"
    raw_gemv = None
    MIN_DIM = 1024

    @classmethod
    def wants(cls, mod) -> bool:
        return _raw_bf16_linear(mod, cls.MIN_DIM, None, cls.MIN_DIM)

    @classmethod
    def adopt(cls, lin: torch.nn.Linear, mode: str) -> "StockLinear":
        """The Linear itself, re-classed in place: the same module object
        with its own Parameters, buffers and hooks (nothing is copied or
        rebuilt), now forwarding through stock_linear under `mode`."""
        lin.__class__ = cls
        lin.stock_gemv = mode
        lin.raw_gemv = None
        return lin

    def forward(self, x):
        return stock_linear(x, self.weight, self.bias, self.stock_gemv, self.raw_gemv)


def install_stock_gemv(model, device, mode: str, raw: str = "stock") -> int:
    """The stock GEMV `mode` onto the tree (swap.py:806-847): every raw
    Linear StockLinear wants is adopted and every StockLinear / RawLinear
    told the mode; under "triton", or "twin" in a codec tree, each also gets
    its raw_gemv_dict. Returns how many modules run a route; nothing off the
    accelerator, or for "linear" without the raw GEMV."""
    if not str(device).startswith("cuda"):
        return 0
    twin = mode == "triton" or (raw == "twin" and codec_tree(model))
    if mode == "linear" and not twin:
        return 0
    done = 0
    for _, parent in list(model.named_modules()):
        for child_name, child in list(parent.named_children()):
            if StockLinear.wants(child):
                child = StockLinear.adopt(child, mode)
                setattr(parent, child_name, child)
            elif isinstance(child, (StockLinear, RawLinear)):
                child.stock_gemv = mode
            else:
                continue
            R, C = (child.out_features, child.in_features) if isinstance(child, StockLinear) else (child.R, child.C)
            child.raw_gemv = raw_gemv_dict(R, C) if twin else None
            done += 1
    return done


class NarrowLinear(torch.nn.Linear):
    """A raw bf16 Linear below the codec's row threshold served by the raw
    GEMV for M <= MC_MAX (swap.py:530-626)."""

    MAX_ROWS = 1024
    MIN_COLS = 1024
    BLOCK = 512
    NUM_WARPS = 4

    @classmethod
    def wants(cls, mod) -> bool:
        return (not eligible(mod) and _raw_bf16_linear(mod, 1, cls.MAX_ROWS, cls.MIN_COLS)
                and mod.weight.shape[1] % 4 == 0)

    @classmethod
    def adopt(cls, lin: torch.nn.Linear) -> "NarrowLinear":
        """The Linear re-classed in place (its own Parameters, no copy)."""
        lin.__class__ = cls
        return lin

    def forward(self, x):
        shape = x.shape
        xm = x.reshape(-1, self.in_features)
        M = xm.shape[0]
        if M > MC_MAX or x.device.type != "cuda":
            return torch.nn.functional.linear(x, self.weight, self.bias)
        y = radix_ops.gemv_narrow(self.weight, xm, self.bias, self.BLOCK, self.NUM_WARPS)
        return y.reshape(*shape[:-1], self.out_features)


def install_narrow(model, device) -> list[tuple[str, tuple[int, int]]]:
    """Every raw Linear NarrowLinear wants, adopted in place; the (name,
    (R, C)) list of what was done (swap.py:613-626). Nothing off the
    accelerator, nothing the codec holds."""
    if not str(device).startswith("cuda"):
        return []
    done = []
    for parent_name, parent in list(model.named_modules()):
        for child_name, child in list(parent.named_children()):
            if NarrowLinear.wants(child):
                setattr(parent, child_name, NarrowLinear.adopt(child))
                done.append((f"{parent_name}.{child_name}" if parent_name else child_name, tuple(child.weight.shape)))
    return done


def eligible(mod) -> bool:
    """Does the codec take this Linear (swap.py:850-854)? A bf16 weight whose
    rows and columns are both at least 1024, columns a multiple of 4. Which
    Linears of a model to hand to the loader is the caller's walk."""
    if not isinstance(mod, torch.nn.Linear):
        return False
    R, C = mod.weight.shape
    return mod.weight.dtype == torch.bfloat16 and C % 4 == 0 and min(R, C) >= 1024


def make_module(pack: dict, bias, device="cuda", row_begin: int = 0, row_end: int | None = None):
    """The loader's one constructor: a pack dict -> the resident module for
    it, by the tensor's own kind (swap.py:900-919). With a row range, the
    module holds that shard of the rows (and of the bias)."""
    if pack.get("codec") == "radix":
        rt = to_device_radix(pack, device, row_begin, row_end)
        if bias is not None and row_end is not None:
            bias = bias[row_begin:row_end]
        return RadixCompressedLinear(rt, bias)
    if pack.get("codec") == "raw":
        rt = to_device_raw(pack, device)
        return RawLinear(rt, bias)
    raise ValueError(f"pack tensor declares codec {pack.get('codec')!r}: not a radix or raw tensor this build serves "
                     "— refusing to build a module for it")
