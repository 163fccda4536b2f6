"""The radix pack tensor: format constants, the encoder and the pack-format-1
reader, mirroring the reference's names so callers read the same.

Reference (file:line in the reference project):
  PROFILES, DEFAULT_BLOCK       src/drinkme/codec/radix.py:13-18
  block_word_bounds             src/drinkme/codec/radix.py:149-171
  pack_array_radix / raw_dict   src/drinkme/codec/radix_pack.py:175-214
  pack_weight_radix             src/drinkme/codec/radix_pack.py:217-236
  padded_palette_words          src/drinkme/codec/radix_pack.py:333-350
  pack_weight_served            src/drinkme/codec/pack.py:107-116
  validate_tensor               src/drinkme/codec/pack.py:210-276
  iter_pack_dir / read tensor   src/drinkme/codec/pack.py:629-693

The encoder is the C library's (dm_pack_plan / dm_pack_encode), which
writes the reference's bytes; the reader reads pack format 1 unchanged.
"""
from __future__ import annotations

import ctypes as ct
import json
import os
import re

import numpy as np

from . import _lib

FORMAT_VERSION = 1
RADIX = "radix"
RAW = "raw"
DEFAULT_BLOCK = 1024
RADIX_BLOCK = DEFAULT_BLOCK
PROFILES = {"gulp": (2, 2, 4, 8), "balanced": (2, 3, 8), "sip": (3, 8)}
PUBLIC_PROFILES = ("sip", "gulp")
DEFAULT_PROFILE = "sip"
MANT, EXP = 7, 8

_ARRAYS_RADIX = ("rx_palette", "rx_offsets", "rx_data")
_SCALARS_RADIX = ("R", "C", "bpw", "codec", "profile", "widths", "block_size")
_ARRAYS_RAW = ("raw_bits",)
_SCALARS_RAW = ("R", "C", "bpw", "codec")


def widths_of(compression_profile: str) -> tuple[int, ...]:
    if compression_profile not in PROFILES:
        raise ValueError(f"unknown profile {compression_profile!r}; one of {tuple(PROFILES)}")
    return PROFILES[compression_profile]


def resolve_compression_profile(explicit: str | None = None) -> str:
    """radix_pack.resolve_compression_profile: explicit, else
    DRINKME_COMPRESSION_PROFILE, else sip."""
    name = explicit or os.environ.get("DRINKME_COMPRESSION_PROFILE", "").strip() or DEFAULT_PROFILE
    if name not in PROFILES:
        raise ValueError(f"unknown profile {name!r}; one of {tuple(PROFILES)}")
    return name


def _cw(n, width):
    return (n * width + 31) // 32


def block_word_bounds(n, mant: int = MANT, exponent: int = EXP, widths=(3, 8)) -> tuple:
    """The fewest and the most uint32 words a block of n weights can take."""
    n = np.asarray(n, dtype=np.int64)
    fixed = _cw(n, mant + 1) + _cw(n, widths[0])
    most = fixed + sum(_cw(n, w) for w in widths[1:-1]) + _cw(n, exponent)
    return fixed, most


def padded_table_bytes(widths) -> int:
    return sum(4 * (((1 << int(w)) + 2) // 4) for w in widths[:-1])


def padded_palette_words(p: dict) -> np.ndarray:
    """Each nonterminal tier's (1 << w) - 1 palette bytes zero-padded to whole
    uint32 words, concatenated in tier order."""
    palette = np.ascontiguousarray(p.get("rx_palette_np", p["rx_palette"]), dtype=np.uint8)
    tables, base = [], 0
    for w in [int(x) for x in p["widths"]][:-1]:
        n = (1 << w) - 1
        t = np.zeros(((n + 3) // 4) * 4, dtype=np.uint8)
        t[:n] = palette[base:base + n]
        tables.append(t.view(np.uint32))
        base += n
    return np.concatenate(tables) if tables else np.empty(0, dtype=np.uint32)


def _ptr(a):
    return a.ctypes.data_as(ct.c_void_p)


def encode_arrays(U: np.ndarray, widths, block_size: int = DEFAULT_BLOCK, threads: int = 0):
    """uint16 [R, C] bf16 bits -> (palette u8 unpadded, offsets u32, data u32)
    as the reference's encoders write them (radix.pack_array's streams for
    any block size; radix_native's for 1024)."""
    U = np.ascontiguousarray(U, dtype=np.uint16)
    if U.ndim != 2 or min(U.shape) < 1:
        raise ValueError("expected a nonempty 2D uint16 array of bf16 bit patterns")
    R, C = U.shape
    w = np.ascontiguousarray([int(x) for x in widths], dtype=np.int32)
    covered = sum((1 << int(x)) - 1 for x in widths[:-1])
    nb = (C + block_size - 1) // block_size
    palette = np.zeros(max(covered, 1), dtype=np.uint8)
    offsets = np.zeros(R * nb + 1, dtype=np.uint32)
    nwords = ct.c_uint64()
    _lib.call("dm_pack_plan", _ptr(U), R, C, _ptr(w), len(w), int(block_size), int(threads), _ptr(palette),
              _ptr(offsets), ct.byref(nwords))
    data = np.zeros(int(nwords.value), dtype=np.uint32)
    _lib.call("dm_pack_encode", _ptr(U), R, C, _ptr(w), len(w), int(block_size), int(threads), _ptr(palette),
              _ptr(offsets), _ptr(data), int(nwords.value))
    return palette[:covered], offsets, data


def decode_pack_device(p: dict, device="cuda"):
    """A radix pack decoded on a GPU straight from its own arrays (the word
    stream and directory copied as they are; dm_decode_pack): uint16 bf16
    bit patterns [R, C] as a CUDA tensor, bit-exact to the source."""
    import torch

    dev = torch.device(device)
    palette = np.ascontiguousarray(p["rx_palette"], dtype=np.uint8)
    offsets = np.ascontiguousarray(p["rx_offsets"], dtype=np.uint32)
    data = np.ascontiguousarray(p["rx_data"], dtype=np.uint32)
    R, C = int(p["R"]), int(p["C"])
    w = np.ascontiguousarray([int(x) for x in p["widths"]], dtype=np.int32)
    d_data = torch.zeros(data.size + 64, dtype=torch.int32, device=dev)  # a zero tail past the last block
    d_data[: data.size].copy_(torch.from_numpy(data.view(np.int32)))
    d_off = torch.from_numpy(offsets.view(np.int32)).to(dev)
    out = torch.empty((R, C), dtype=torch.int16, device=dev)
    stream = ct.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    _lib.call("dm_decode_pack", _ptr(palette), palette.size, _ptr(offsets), offsets.size, data.size, R, C, _ptr(w),
              len(w), int(p.get("block_size", DEFAULT_BLOCK)), ct.c_void_p(d_data.data_ptr()),
              ct.c_void_p(d_off.data_ptr()), ct.c_void_p(out.data_ptr()), stream)
    return out


def encode_arrays_device(bits, widths, block_size: int = DEFAULT_BLOCK):
    """encode_arrays on the GPU: `bits` is a CUDA tensor of uint16 (or int16)
    bf16 patterns [R, C]; the exponent histogram, the per-block word counts
    and the payload are computed on its device (dm_pack_plan_device /
    dm_pack_encode_device). Returns the same (palette, offsets, data) numpy
    arrays, byte for byte."""
    import torch

    if not isinstance(bits, torch.Tensor) or bits.device.type != "cuda":
        raise TypeError("encode_arrays_device: expected a CUDA tensor of bf16 bit patterns")
    if bits.dim() != 2 or min(bits.shape) < 1 or bits.element_size() != 2 or bits.is_floating_point():
        raise ValueError("expected a nonempty 2D uint16 array of bf16 bit patterns")
    bits = bits.contiguous()
    R, C = bits.shape
    w = np.ascontiguousarray([int(x) for x in widths], dtype=np.int32)
    covered = sum((1 << int(x)) - 1 for x in widths[:-1])
    nb = (C + block_size - 1) // block_size
    palette = np.zeros(max(covered, 1), dtype=np.uint8)
    offsets = np.zeros(R * nb + 1, dtype=np.uint32)
    nwords = ct.c_uint64()
    stream = ct.c_void_p(torch.cuda.current_stream(bits.device).cuda_stream)
    _lib.call("dm_pack_plan_device", ct.c_void_p(bits.data_ptr()), R, C, _ptr(w), len(w), int(block_size),
              _ptr(palette), _ptr(offsets), ct.byref(nwords), stream)
    n = int(nwords.value)
    data = torch.empty(max(n, 1), dtype=torch.int32, device=bits.device)
    _lib.call("dm_pack_encode_device", ct.c_void_p(bits.data_ptr()), R, C, _ptr(w), len(w), int(block_size),
              _ptr(palette), _ptr(offsets), ct.c_void_p(data.data_ptr()), n, stream)
    # the payload comes back through a pinned buffer kept for the next call
    # (a fresh pageable array would fault in every page during the copy)
    host = np.empty(n, dtype=np.uint32)
    pinned = _pinned_staging(n * 4)
    done = 0
    while done < n:
        k = min(n - done, pinned.numel() // 4)
        pinned[: k * 4].view(torch.int32).copy_(data[done: done + k], non_blocking=True)
        torch.cuda.current_stream(bits.device).synchronize()
        host[done: done + k] = pinned[: k * 4].numpy().view(np.uint32)
        done += k
    return palette[:covered], offsets, host


_PINNED = None


def _pinned_staging(nbytes: int):
    """A pinned host buffer of up to 64 MiB, reused across calls."""
    import torch

    global _PINNED
    want = min(max(nbytes, 1 << 20), 64 << 20)
    if _PINNED is None or _PINNED.numel() < want:
        _PINNED = torch.empty(want, dtype=torch.uint8, pin_memory=True)
    return _PINNED


def pack_array_radix_device(bits, compression_profile: str, block_size: int = RADIX_BLOCK) -> dict | None:
    """pack_array_radix for bits already on a GPU (encode_arrays_device): the
    same dict, byte for byte, or None when radix would not compress."""
    widths = widths_of(compression_profile)
    palette, offsets, data = encode_arrays_device(bits, widths, block_size)
    R, C = bits.shape
    if _would_expand(palette, offsets, data, widths, R * C * 2):
        return None
    stored = palette.nbytes + offsets.nbytes + data.nbytes
    return {"rx_palette": palette, "rx_offsets": offsets, "rx_data": data, "R": int(R), "C": int(C),
            "bpw": 8.0 * stored / (R * C), "codec": RADIX, "profile": compression_profile,
            "widths": list(widths), "block_size": int(block_size)}


def _would_expand(palette, offsets, data, widths, nbytes: int) -> bool:
    """radix_pack._would_expand: stored OR device bytes reaching the raw
    plane's size means no compression."""
    stored = palette.nbytes + offsets.nbytes + data.nbytes
    device = data.nbytes + offsets.nbytes + padded_table_bytes(widths)
    return max(stored, device) >= nbytes


def pack_array_radix(U: np.ndarray, compression_profile: str, block_size: int = RADIX_BLOCK,
                     threads: int = 0) -> dict | None:
    """uint16 [R, C] bf16 bits -> the radix tensor dict, or None when radix
    would not compress this tensor (the caller stores it raw)."""
    U = np.ascontiguousarray(U, dtype=np.uint16)
    if U.ndim != 2 or min(U.shape) < 1:
        raise ValueError("pack_array_radix: need a nonempty 2D uint16 array")
    widths = widths_of(compression_profile)
    palette, offsets, data = encode_arrays(U, widths, block_size, threads)
    if _would_expand(palette, offsets, data, widths, U.nbytes):
        return None
    R, C = U.shape
    stored = palette.nbytes + offsets.nbytes + data.nbytes
    return {"rx_palette": palette, "rx_offsets": offsets, "rx_data": data, "R": int(R), "C": int(C),
            "bpw": 8.0 * stored / (R * C), "codec": RADIX, "profile": compression_profile,
            "widths": list(widths), "block_size": int(block_size)}


def raw_dict(U: np.ndarray) -> dict:
    U = np.ascontiguousarray(U, dtype=np.uint16)
    if U.ndim != 2 or min(U.shape) < 1:
        raise ValueError("raw_dict: need a nonempty 2D uint16 array")
    R, C = U.shape
    return {"raw_bits": U, "R": int(R), "C": int(C), "bpw": 16.0, "codec": RAW}


def bits_of(w_bf16) -> np.ndarray:
    import torch

    if w_bf16.dtype != torch.bfloat16:
        raise TypeError(f"{w_bf16.dtype} is not bf16 — the codec packs bf16 bits as released and never converts")
    return w_bf16.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def pack_weight_radix(w_bf16, compression_profile: str, name: str | None = None, threads: int = 0) -> dict:
    """One tensor: the radix dict, or the raw dict when radix would expand it."""
    U = bits_of(w_bf16)
    p = pack_array_radix(U, compression_profile, threads=threads)
    return raw_dict(U) if p is None else p


def pack_weight_served(w_bf16, name: str | None = None, compression_profile: str | None = None) -> dict:
    """pack.pack_weight_served: the resolved profile (sip by default)."""
    p = pack_weight_radix(w_bf16, resolve_compression_profile(compression_profile), name=name)
    p["format_version"] = FORMAT_VERSION
    return p


def is_radix_pack(p: dict) -> bool:
    return p.get("codec") == RADIX


def is_raw_pack(p: dict) -> bool:
    return p.get("codec") == RAW


# ------------------------------------------------------------ the reader --

MAX_TENSOR_WEIGHTS = 1 << 33
_TENSOR_FILE = re.compile(r"t\d{4,}\.npz\Z")


def _validate_radix_descriptors(name: str, p: dict) -> None:
    """radix.validate (radix.py:174-238) over the dict: the checks and
    messages the C loader (dm_tensor_create) applies, here on the host before
    anything is allocated."""
    pal = np.ascontiguousarray(p["rx_palette"], dtype=np.uint8)
    off = np.ascontiguousarray(p["rx_offsets"], dtype=np.uint32)
    data = np.ascontiguousarray(p["rx_data"], dtype=np.uint32)
    w = np.ascontiguousarray([int(x) for x in p["widths"]], dtype=np.int32)
    R, C, B = int(p["R"]), int(p["C"]), int(p["block_size"])
    if B < 32 or B > 4096 or B & (B - 1):
        raise ValueError("invalid radix block size")
    covered = sum((1 << int(x)) - 1 for x in w[:-1])
    if pal.size != covered or len(np.unique(pal)) != covered:
        raise ValueError("invalid radix palette entries")
    nb = R * ((C + B - 1) // B)
    if off.size != nb + 1 or off[0] != 0 or int(off[-1]) != data.size or np.any(off[1:] <= off[:-1]):
        raise ValueError("invalid radix block offsets")
    per_row = (C + B - 1) // B
    n = np.minimum(B, C - np.arange(nb, dtype=np.int64) % per_row * B)
    length = off[1:].astype(np.int64) - off[:-1].astype(np.int64)
    fewest, most = block_word_bounds(n, MANT, EXP, tuple(int(x) for x in w))
    short = np.flatnonzero(length < fewest)
    if short.size:
        i = int(short[0])
        raise ValueError(f"invalid radix block offsets: block {i} holds {int(length[i])} word(s), fewer than the "
                         f"{int(fewest[i])} its literal plane and first tier take for {int(n[i])} weights")
    long_ = np.flatnonzero(length > most)
    if long_.size:
        i = int(long_[0])
        raise ValueError(f"invalid radix block offsets: block {i} holds {int(length[i])} words, more than the "
                         f"{int(most[i])} any block of {int(n[i])} weights can use")


def validate_tensor(name: str, p: dict) -> None:
    """pack.validate_tensor: the descriptor gate every loader goes through."""
    kind = p.get("codec") or "?"
    R, C = p.get("R"), p.get("C")
    if type(R) is not int or type(C) is not int or R <= 0 or C <= 0:
        raise ValueError(f"pack tensor {name} ({kind}): R, C must be positive ints, got {R!r}, {C!r}")
    if R * C > MAX_TENSOR_WEIGHTS:
        raise ValueError(f"pack tensor {name} ({kind}): R x C = {R:,} x {C:,} is {R * C:,} weights, "
                         f"more than the {MAX_TENSOR_WEIGHTS:,} this loader will allocate for")
    if kind == RADIX:
        widths = p.get("widths")
        if (not isinstance(widths, (list, tuple)) or len(widths) < 2
                or any(isinstance(w, bool) or not isinstance(w, (int, np.integer)) for w in widths)):
            raise ValueError(f"pack tensor {name} (radix): widths {widths!r} is not a list of 2+ ints")
        widths = tuple(int(w) for w in widths)
        if p.get("block_size") != RADIX_BLOCK:
            raise ValueError(f"pack tensor {name} (radix): block_size {p.get('block_size')!r} — the served kernels "
                             f"walk {RADIX_BLOCK}-weight blocks only")
        if len(widths) > 4:
            raise ValueError(f"pack tensor {name} (radix): widths {list(widths)} is {len(widths)} tiers; "
                             "the scheduled decoder's block header holds at most four (three nonterminal)")
        if any(w > 4 or w < 1 for w in widths[:-1]):
            raise ValueError(f"pack tensor {name} (radix): widths {list(widths)} — a nonterminal tier "
                             "must be 1..4 bits (one byte of the block header per tier)")
        if widths[-1] != 8:
            raise ValueError(f"pack tensor {name} (radix): widths {list(widths)} — the terminal tier is "
                             "the 8-bit bf16 exponent")
        if p.get("profile") not in PROFILES:
            raise ValueError(f"pack tensor {name} (radix): profile {p.get('profile')!r} is not one this "
                             f"drinkme packs or serves ({' | '.join(PUBLIC_PROFILES)})")
        for key in _ARRAYS_RADIX:
            if key not in p:
                raise ValueError(f"pack tensor {name} (radix): no {key} array")
        try:
            _validate_radix_descriptors(name, p)
        except ValueError as e:
            raise ValueError(f"pack tensor {name} (radix): {e}") from None
    elif kind == RAW:
        bits = p.get("raw_bits")
        if bits is None:
            raise ValueError(f"pack tensor {name} (raw): no raw_bits array")
        bits = np.asarray(bits)
        if bits.dtype != np.uint16:
            raise ValueError(f"pack tensor {name} (raw): raw_bits dtype {bits.dtype}, not uint16")
        if bits.shape != (R, C):
            raise ValueError(f"pack tensor {name} (raw): raw_bits is {bits.shape}, not [R, C] = ({R}, {C})")
    else:
        raise ValueError(f"pack tensor {name} declares codec {p.get('codec')!r}, which this build does not "
                         f"implement (knows {RADIX!r} and {RAW!r}) — refusing to load.")


def _tensor_file(path: str, name: str, fn) -> str:
    if not isinstance(fn, str) or not _TENSOR_FILE.fullmatch(fn) or os.path.basename(fn) != fn:
        raise ValueError(f"{path}/meta.json: tensor {name!r} names file {fn!r}; a pack file is a "
                         "bare basename of the form t0000.npz — refusing to open it")
    root = os.path.realpath(path)
    fp = os.path.realpath(os.path.join(path, fn))
    if os.path.dirname(fp) != root:
        raise ValueError(f"{path}/meta.json: tensor {name!r}'s file {fn!r} resolves to {fp}, outside "
                         "the pack directory — refusing to open it")
    return os.path.join(path, fn)


def _check_format_version(meta: dict, path: str) -> int:
    v = meta.get("formatVersion")
    if v != FORMAT_VERSION:
        raise ValueError(f"{path}: pack format {v!r} is not readable by this build (reads {FORMAT_VERSION})")
    prof = meta.get("profile")
    if prof is not None and prof not in PROFILES:
        raise ValueError(f"{path}: pack profile {prof!r} is not one this build reads ({tuple(PROFILES)})")
    return int(v)


def read_tensor_file(path: str, name: str, fn) -> dict:
    with np.load(_tensor_file(path, name, fn)) as z:
        sc = json.loads(str(z["scalars"][0]))
        codec = sc.get("codec")
        keys = _ARRAYS_RADIX if codec == RADIX else _ARRAYS_RAW if codec == RAW else None
        if keys is None:
            raise ValueError(f"pack tensor {name} declares codec {codec!r}, which this build does not implement "
                             f"(knows {RADIX!r} and {RAW!r}) — refusing to load.")
        R, C = sc.get("R"), sc.get("C")
        sizes = {i.filename: i.file_size for i in z.zip.infolist()}
        for k in keys:
            if k + ".npy" not in sizes:
                raise ValueError(f"pack tensor {name} ({codec}): the npz holds no {k}.npy")
            if isinstance(R, int) and isinstance(C, int) and sizes[k + ".npy"] > 2 * R * C + 4096:
                raise ValueError(f"pack tensor {name} ({codec}): {k}.npy is {sizes[k + '.npy']:,} bytes, more "
                                 f"than the 2 x R x C the tensor's bf16 plane takes — refusing to allocate it")
        p = {k: np.asarray(z[k]) for k in keys}
        p.update(sc)
    p["format_version"] = FORMAT_VERSION
    validate_tensor(name, p)
    return p


def iter_pack_dir(path: str, skip: tuple[str, ...] | None = None):
    """Yield (tensor_name, pack_dict) one tensor at a time, each validated."""
    with open(os.path.join(path, "meta.json")) as f:
        meta = json.load(f)
    _check_format_version(meta, path)
    for name, fn in meta["tensors"].items():
        if skip is not None and any(name == s or name.startswith(s + ".") for s in skip):
            continue
        yield name, read_tensor_file(path, name, fn)


def save_pack_dir(path: str, tensors: dict, meta: dict) -> None:
    """Write a pack-format-1 directory: meta.json + one npz per tensor (the
    reference's container layout, pack.py:467-579; for tests and tools)."""
    os.makedirs(path, exist_ok=True)
    names = {}
    for i, (name, p) in enumerate(tensors.items()):
        fn = f"t{i:04d}.npz"
        names[name] = fn
        arrays = _ARRAYS_RADIX if p.get("codec") == RADIX else _ARRAYS_RAW
        scalars = _SCALARS_RADIX if p.get("codec") == RADIX else _SCALARS_RAW
        np.savez(os.path.join(path, fn), **{k: p[k] for k in arrays},
                 scalars=np.array([json.dumps({k: p[k] for k in scalars})]))
    full = {"formatVersion": FORMAT_VERSION, "tensors": names, **meta}
    full.setdefault("profile", next((str(p["profile"]) for p in tensors.values() if is_radix_pack(p)),
                                    DEFAULT_PROFILE))
    with open(os.path.join(path, "meta.json"), "w") as f:
        json.dump(full, f, indent=2)
