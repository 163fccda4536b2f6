"""TEST INFRASTRUCTURE — the CPU oracle for drinkme's radix hot path.

Only tests/, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
may import this module, and only as the checker (or, for the CPU baseline,
as the timed reference). The product package ``drinkme_b200`` never imports
it: its decode and linear paths run on the GPU and raise when the CUDA
extension is missing.

Two CPU implementations live here:

* ``liboracle.so`` — our plain-C restatement of the reference's algorithm
  (radix_oracle.c cites the reference file:line for each function):
  validate, strict decode, the gulp schedule, and the float64 linear that
  bench/radix_gemv_bitpin.py:181-186 gates against.
* ``_ref/radix_native.so`` — the reference's own native codec
  (src/drinkme/codec/radix_native.cpp), compiled from its sources by
  oracle/Makefile when they are present. Its decode (op 2) is what the
  reference's CPU route runs (radix_native.py:220-259, called from
  radix_pack.decode_back_radix and swap.CompressedLinear's "cpu" route).

Pack dicts are the reference's tensor dicts (radix_pack.py:9-21):
``rx_palette`` u8 (unpadded), ``rx_offsets`` u32 [R*NB+1], ``rx_data`` u32,
``R``, ``C``, ``widths``, ``block_size``.
"""
from __future__ import annotations

import ctypes as ct
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None
_REF = None


class OracleError(ValueError):
    pass


def library():
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "_build", "liboracle.so")
        if not os.path.exists(path):
            raise OracleError(f"oracle library missing: run `make -C oracle` ({path})")
        lib = ct.CDLL(path)
        p = ct.c_void_p
        i64 = ct.c_int64
        lib.oracle_word_bounds.argtypes = [i64, p, ct.c_int32, p, p]
        lib.oracle_validate.argtypes = [i64, i64, i64, p, ct.c_int32, p, i64, p, i64, i64, p, ct.c_size_t]
        lib.oracle_decode.argtypes = [i64, i64, i64, p, ct.c_int32, p, i64, p, i64, p, i64, p, p, ct.c_size_t]
        lib.oracle_schedule.argtypes = [i64, i64, i64, p, ct.c_int32, p, p, i64, p]
        lib.oracle_linear_f64.argtypes = [i64, i64, i64, p, p, p, p]
        for fn in ("oracle_word_bounds", "oracle_validate", "oracle_decode", "oracle_schedule",
                   "oracle_linear_f64"):
            getattr(lib, fn).restype = ct.c_int
        _LIB = lib
    return _LIB


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ct.c_void_p)


def _arrays(p: dict):
    pal = np.ascontiguousarray(p["rx_palette"], dtype=np.uint8)
    off = np.ascontiguousarray(p["rx_offsets"], dtype=np.uint32)
    data = np.ascontiguousarray(p["rx_data"], dtype=np.uint32)
    if "NW" in p:
        data = data[: int(p["NW"])]
    widths = np.ascontiguousarray([int(w) for w in p["widths"]], dtype=np.int32)
    return pal, off, data, widths


def word_bounds(n: int, widths) -> tuple[int, int]:
    """radix.py:149-171 for one block of n weights (bf16: 7 + 1 literal bits)."""
    w = np.ascontiguousarray([int(x) for x in widths], dtype=np.int32)
    a, b = ct.c_int64(), ct.c_int64()
    library().oracle_word_bounds(int(n), _ptr(w), len(w), ct.byref(a), ct.byref(b))
    return a.value, b.value


def validate(p: dict) -> None:
    pal, off, data, widths = _arrays(p)
    err = ct.create_string_buffer(512)
    rc = library().oracle_validate(int(p["R"]), int(p["C"]), int(p["block_size"]), _ptr(widths), len(widths),
                                   _ptr(pal), pal.size, _ptr(off), off.size, data.size, err, 512)
    if rc:
        raise OracleError(err.value.decode())


def decode(p: dict) -> np.ndarray:
    """The pack dict's uint16 [R, C] bits (radix.py:241-278, strict)."""
    pal, off, data, widths = _arrays(p)
    R, C = int(p["R"]), int(p["C"])
    out = np.zeros((R, C), dtype=np.uint16)
    err = ct.create_string_buffer(512)
    rc = library().oracle_decode(R, C, int(p["block_size"]), _ptr(widths), len(widths), _ptr(pal), pal.size,
                                 _ptr(off), off.size, _ptr(data), data.size, _ptr(out), err, 512)
    if rc:
        raise OracleError(err.value.decode())
    return out


def schedule(p: dict) -> np.ndarray | None:
    """radix_pack.schedule_np: None for two tiers, else uint16 per block."""
    pal, off, data, widths = _arrays(p)
    if len(widths) <= 2:
        return None
    R, C, B = int(p["R"]), int(p["C"]), int(p["block_size"])
    nb = R * ((C + B - 1) // B)
    out = np.zeros(nb, dtype=np.uint16)
    library().oracle_schedule(R, C, B, _ptr(widths), len(widths), _ptr(off), _ptr(data), data.size, _ptr(out))
    return out


def linear_f64(x: np.ndarray, bits: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """(x @ W^T, |x| @ |W|^T) in float64; x [M, C] any float dtype, bits
    uint16 [R, C] bf16 patterns."""
    x = np.ascontiguousarray(np.atleast_2d(x), dtype=np.float64)
    bits = np.ascontiguousarray(bits, dtype=np.uint16)
    M, C = x.shape
    R = bits.shape[0]
    y = np.zeros((M, R), dtype=np.float64)
    a = np.zeros((M, R), dtype=np.float64)
    library().oracle_linear_f64(M, R, C, _ptr(x), _ptr(bits), _ptr(y), _ptr(a))
    return y, a


def gemv_bound(x: np.ndarray, bits: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """The reference's per-element gate (bench/radix_gemv_bitpin.py:182):
    returns (y64, bound) with bound = 2e-6 * |x|.|W| + 1e-7."""
    y, a = linear_f64(x, bits)
    return y, 2e-6 * a + 1e-7


# ---------------------------------------------------------------- numpy --
# An independent second restatement (vectorised per block), used by the
# tests to cross-check the C oracle on small tensors.


def _get(stream: np.ndarray, start: int, count: int, width: int):
    bit = np.arange(count, dtype=np.int64) * width
    words = (count * width + 31) // 32
    if start + words > len(stream):
        raise OracleError("truncated radix stream")
    v = stream[start + bit // 32].astype(np.uint64) >> (bit % 32).astype(np.uint64)
    cross = bit % 32 + width > 32
    if cross.any():
        v[cross] |= stream[start + bit[cross] // 32 + 1].astype(np.uint64) << (32 - bit[cross] % 32).astype(np.uint64)
    return (v & ((1 << width) - 1)).astype(np.uint32), start + words


def decode_numpy(p: dict) -> np.ndarray:
    pal, off, data, widths = _arrays(p)
    R, C, B = int(p["R"]), int(p["C"]), int(p["block_size"])
    per_row = (C + B - 1) // B
    out = np.zeros((R, C), dtype=np.uint16)
    for r in range(R):
        for b in range(per_row):
            blk = r * per_row + b
            n = min(B, C - b * B)
            s = data[int(off[blk]):int(off[blk + 1])]
            lit, pos = _get(s, 0, n, 8)
            exps = np.zeros(n, dtype=np.uint32)
            active = np.arange(n)
            base = 0
            for w in widths[:-1]:
                code, pos = _get(s, pos, len(active), int(w))
                esc = (1 << int(w)) - 1
                done = code != esc
                exps[active[done]] = pal[base + code[done]]
                active = active[~done]
                base += esc
            exps[active], pos = _get(s, pos, len(active), 8)
            if pos != len(s):
                raise OracleError("radix block has trailing words")
            out[r, b * B:b * B + n] = (lit & 0x7F) | ((lit >> 7) << 15) | (exps << 7)
    return out


# ------------------------------------------------------ the reference's --


def reference_native():
    """The reference's own radix_native.so (compiled into oracle/_ref/ from
    its sources), or None when it was not built."""
    global _REF
    if _REF is None:
        path = os.path.join(_HERE, "_ref", "radix_native.so")
        if not os.path.exists(path):
            _REF = False
            return None
        lib = ct.CDLL(path)
        fn = lib.radix_native
        u32, u64, p = ct.c_uint32, ct.c_uint64, ct.c_void_p
        fn.argtypes = [u32, p, u64, u64, u64, u64, u32, u32, p, u32, p, p, p, u64, u64, u64, p, p, u64]
        fn.restype = ct.c_int
        _REF = lib
    return _REF or None


def _ref_tables(pal: np.ndarray, widths) -> np.ndarray:
    """The per-tier word-padded palette the native library indexes
    (radix_native.py:187-192 padded_table_bytes, 236-242)."""
    size = sum(4 * (((1 << int(w)) + 2) // 4) for w in widths[:-1])
    t = np.zeros(size, dtype=np.uint8)
    at = base = 0
    for w in widths[:-1]:
        n = (1 << int(w)) - 1
        t[at:at + n] = pal[base:base + n]
        at += ((n + 3) // 4) * 4
        base += n
    return t


def reference_decode(p: dict, first: int = 0, rows: int | None = None, out: np.ndarray | None = None) -> np.ndarray:
    """Rows [first, first+rows) decoded by the reference's native library
    (op 2, 1024-weight blocks only), single call = single thread."""
    lib = reference_native()
    if lib is None:
        raise OracleError("the reference's native codec is not built (oracle/_ref)")
    pal, off, data, widths = _arrays(p)
    R, C = int(p["R"]), int(p["C"])
    if int(p["block_size"]) != 1024:
        raise OracleError("the reference's native codec reads 1024-weight blocks only")
    rows = R - first if rows is None else rows
    tables = _ref_tables(pal, widths)
    w = np.ascontiguousarray(widths, dtype=np.uint32)
    if out is None:
        out = np.empty((rows, C), dtype=np.uint16)
    err = ct.create_string_buffer(1024)
    res = ct.c_uint64()
    nb = (C + 1023) // 1024
    rc = lib.radix_native(2, _ptr(out), R, C, R, nb, 7, 8, _ptr(w), len(w), _ptr(tables), _ptr(off), _ptr(data),
                          data.size, first, rows, ct.byref(res), err, 1024)
    if rc:
        raise OracleError("reference native: " + err.value.decode())
    return out


def reference_encode(U: np.ndarray, widths=(3, 8)) -> dict:
    """uint16 [R, C] bf16 bits -> a pack dict made by the reference's own
    native encoder (op 0 plan, op 1 encode; radix_native.py:195-217 drives
    the same two calls), 1024-weight blocks. The palette comes back padded
    per tier and is unpadded here as the reference's wrapper does."""
    lib = reference_native()
    if lib is None:
        raise OracleError("the reference's native codec is not built (oracle/_ref)")
    U = np.ascontiguousarray(U, dtype=np.uint16)
    R, C = U.shape
    nb = (C + 1023) // 1024
    w = np.ascontiguousarray([int(v) for v in widths], dtype=np.uint32)
    tables = np.zeros(sum(4 * (((1 << int(v)) + 2) // 4) for v in widths[:-1]), dtype=np.uint8)
    offsets = np.zeros(R * nb + 1, dtype=np.uint32)
    err = ct.create_string_buffer(1024)
    res = ct.c_uint64()

    def op(code, data, nwords):
        rc = lib.radix_native(code, _ptr(U), R, C, R, nb, 7, 8, _ptr(w), len(w), _ptr(tables), _ptr(offsets),
                              None if data is None else _ptr(data), nwords, 0, 0, ct.byref(res), err, 1024)
        if rc:
            raise OracleError("reference native: " + err.value.decode())
        return res.value

    words = op(0, None, 0)
    data = np.zeros(words, dtype=np.uint32)
    op(1, data, data.size)
    parts, at = [], 0
    for v in widths[:-1]:
        n = (1 << int(v)) - 1
        parts.append(tables[at:at + n])
        at += ((n + 3) // 4) * 4
    return {"rx_palette": np.concatenate(parts).astype(np.uint8), "rx_offsets": offsets, "rx_data": data,
            "R": R, "C": C, "widths": tuple(int(v) for v in widths), "block_size": 1024, "codec": "radix"}


def reference_decode_threads(p: dict, workers: int) -> np.ndarray:
    """The reference's decode with `workers` threads (radix_native.py:245-259:
    row ranges of about R / (4 workers) rows, one native call each; ctypes
    releases the GIL during a call)."""
    from concurrent.futures import ThreadPoolExecutor

    R, C = int(p["R"]), int(p["C"])
    out = np.empty((R, C), dtype=np.uint16)
    if workers <= 1 or R < 2 * workers:
        return reference_decode(p, 0, R, out)
    step = -(-R // (4 * workers))
    ranges = [(a, min(step, R - a)) for a in range(0, R, step)]
    with ThreadPoolExecutor(max_workers=workers) as ex:
        list(ex.map(lambda r: reference_decode(p, r[0], r[1], out[r[0]:r[0] + r[1]]), ranges))
    return out
