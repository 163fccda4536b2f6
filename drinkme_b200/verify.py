"""Decode-and-hash verification of packed tensors, the GPU side of the
reference's upstream verification (src/drinkme/upstream.py; the procedure
of docs/pack-format.md:327-378): a checkpoint file is rebuilt as a sequence
of parts — raw bytes (a safetensors header, a tensor stored as is) and
packed tensors decoded to their BF16 bits — and streamed into SHA-256
without being written out; the digest is compared with the one the
checkpoint's publisher lists for the file.

Here a producer thread copies each radix pack to the GPU as it is, decodes
it there straight from its own arrays (dm_decode_pack) and copies the bits
into one of a few pinned host buffers on a side stream, several parts ahead; the calling thread
hashes the parts in file order as their copies land. SHA-256 of one file is
sequential, so the hash sets the pace once the decode keeps ahead of it.
Fetching digests and reading pack directories are the caller's (the
reference's Hub and file handling are not part of this package).
verify_files hashes several files at once (a thread each: one file's
SHA-256 is sequential, a checkpoint's shards are not).
"""
from __future__ import annotations

import hashlib
import queue
from concurrent.futures import ThreadPoolExecutor
import threading
import time

import numpy as np
import torch

from . import codec

_AHEAD = 3  # pinned buffers: parts decoded and copied ahead of the hash


def _part_bytes(part) -> int:
    if isinstance(part, (bytes, bytearray, memoryview)):
        return len(part)
    return int(part["R"]) * int(part["C"]) * 2


def rebuild_sha256(parts, device="cuda") -> dict:
    """SHA-256 of the concatenation of `parts`, in order: bytes-like parts
    as they are; a raw tensor dict's bits (little-endian uint16) as stored; a
    radix tensor dict decoded on `device` to its BF16 bits. Returns
    {"sha256", "bytes", "seconds", "gbs"}."""
    dev = torch.device(device)
    if dev.type != "cuda":
        raise ValueError("rebuild_sha256 decodes on a CUDA device")
    parts = list(parts)
    for part in parts:
        if not isinstance(part, (bytes, bytearray, memoryview)) and part.get("codec") not in (codec.RADIX, codec.RAW):
            raise ValueError(f"rebuild_sha256: a part of codec {part.get('codec')!r} is neither radix nor raw")
    biggest = max([_part_bytes(p) for p in parts if isinstance(p, dict) and p.get("codec") == codec.RADIX],
                  default=0)
    free: queue.Queue = queue.Queue()
    for _ in range(_AHEAD if biggest else 0):
        free.put(torch.empty(biggest // 2, dtype=torch.int16, pin_memory=True))
    ready: queue.Queue = queue.Queue(maxsize=_AHEAD + 1)
    failure = []

    def produce():
        try:
            torch.cuda.set_device(dev)
            side = torch.cuda.Stream(dev)
            for part in parts:
                if isinstance(part, dict) and part.get("codec") == codec.RADIX:
                    buf = free.get()
                    n = int(part["R"]) * int(part["C"])
                    with torch.cuda.stream(side):
                        bits = codec.decode_pack_device(part, dev)
                        buf[:n].copy_(bits.reshape(-1), non_blocking=True)
                        ev = torch.cuda.Event()
                        ev.record(side)
                    ready.put(("radix", buf, n, ev, bits))
                    del bits
                else:
                    ready.put(("host", part))
        except BaseException as e:  # noqa: BLE001 - reported on the calling thread
            failure.append(e)
            ready.put(("error",))

    h = hashlib.sha256()
    t0 = time.perf_counter()
    worker = threading.Thread(target=produce, daemon=True)
    worker.start()
    try:
        for _ in parts:
            item = ready.get()
            if item[0] == "error":
                raise failure[0]
            if item[0] == "host":
                part = item[1]
                if isinstance(part, (bytes, bytearray, memoryview)):
                    h.update(part)
                else:
                    h.update(np.ascontiguousarray(part["raw_bits"], dtype=np.uint16).tobytes())
                continue
            _, buf, n, ev, rt = item
            ev.synchronize()
            h.update(memoryview(buf[:n].numpy()).cast("B"))
            del rt
            free.put(buf)
    finally:
        while worker.is_alive():  # a failed hash: let the producer finish its puts
            try:
                item = ready.get(timeout=0.05)
            except queue.Empty:
                continue
            if item[0] == "radix":
                free.put(item[1])
        worker.join()
    secs = time.perf_counter() - t0
    total = sum(_part_bytes(p) for p in parts)
    return {"sha256": h.hexdigest(), "bytes": total, "seconds": secs, "gbs": total / secs * 1e-9 if secs > 0 else 0.0}


def verify_parts(parts, expected_sha256: str, device="cuda") -> str:
    """'MATCH' when the rebuilt file hashes to `expected_sha256`, else
    'MISMATCH' (the reference's verdicts for a covered file)."""
    got = rebuild_sha256(parts, device)["sha256"]
    return "MATCH" if got == expected_sha256.lower() else "MISMATCH"


def verify_files(files, device="cuda", workers: int = 4) -> list[dict]:
    """verify_parts over several files at once: `files` is a sequence of
    (parts, expected_sha256); returns, per file, {"verdict", "sha256",
    "bytes", "seconds"}."""
    def one(item):
        parts, want = item
        r = rebuild_sha256(parts, device)
        r["verdict"] = "MATCH" if r["sha256"] == want.lower() else "MISMATCH"
        return r

    files = list(files)
    with ThreadPoolExecutor(max_workers=max(1, min(workers, len(files)))) as pool:
        return list(pool.map(one, files))
