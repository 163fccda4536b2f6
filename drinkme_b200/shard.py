"""Row sharding of packed linears across the GPUs of one box.

Every 1024-weight block belongs to one row and decodes on its own, so a
radix linear splits by output rows with no exchange inside the GEMV: rank k
of N loads rows [r0_k, r1_k) (the loader slices the block directory and
payload, dm_tensor_create's row range) and computes its slice [M, R/N] of
the output. The one exchange is an all-gather of the slices over NVLink
(NCCL), so every rank holds the full [M, R] output for the next layer.

The reference has no multi-GPU code; the split and the gather are this
package's (the row shard is the reference's own loader applied to a slice of
its directory: offsets[r0*NB : r1*NB + 1] rebased, the payload words
between, the same palette).
"""
from __future__ import annotations

import torch

from . import radix_ops, swap
from .tensor import device_view


def row_range(R: int, rank: int, world: int, align: int = 16) -> tuple[int, int]:
    """Rank `rank`'s rows of R split over `world` ranks: equal shards of
    ceil(R / world) rows rounded up to `align` (whole 16-row units), the last
    shard taking what is left (possibly nothing)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"row_range: rank {rank} outside a world of {world}")
    per = -(-R // world)
    per = -(-per // align) * align
    r0 = min(R, rank * per)
    r1 = min(R, r0 + per)
    return r0, r1


def shard_rows_padded(R: int, world: int, align: int = 16) -> int:
    """The rows every rank's gather slot holds (the largest shard)."""
    return row_range(R, 0, world, align)[1]


def gather_rows(local: torch.Tensor, R: int, world: int, group=None, out: torch.Tensor | None = None,
                work: torch.Tensor | None = None) -> torch.Tensor:
    """All-gather the [M, rows_k] output slices of a row-sharded linear into
    the full [M, R] output on every rank (NCCL all_gather_into_tensor over
    equal slots of the largest shard, then one re-layout when M > 1 or the
    shards are uneven)."""
    import torch.distributed as dist

    M, rk = local.shape
    per = shard_rows_padded(R, world)
    if work is None:
        work = torch.empty((world, M, per), dtype=local.dtype, device=local.device)
    if rk == per:
        src = local
    else:
        src = torch.zeros((M, per), dtype=local.dtype, device=local.device)
        src[:, :rk] = local
    dist.all_gather_into_tensor(work.view(world * M, per), src.contiguous(), group=group)
    if M == 1 and per * world == R:
        full = work.view(1, R)
        if out is not None:
            out.copy_(full)
            return out
        return full
    full = work.permute(1, 0, 2).reshape(M, world * per)[:, :R]
    if out is not None:
        out.copy_(full)
        return out
    return full.contiguous()


class ShardedRadixLinear(torch.nn.Module):
    """A radix linear whose rows are split over the ranks of `group`: this
    rank's shard through the fused decode + GEMV, then the all-gather."""

    def __init__(self, pack: dict, bias, device, rank: int, world: int, group=None):
        super().__init__()
        self.R, self.C = int(pack["R"]), int(pack["C"])
        self.rank, self.world, self.group = rank, world, group
        r0, r1 = row_range(self.R, rank, world)
        self.rows = (r0, r1)
        self.local = None
        if r1 > r0:
            self.local = swap.make_module(pack, bias, device, r0, r1)

    def forward(self, x):
        shape = x.shape
        xm = x.reshape(-1, self.C)
        M = xm.shape[0]
        if self.local is not None:
            y = self.local(xm)
        else:
            y = torch.zeros((M, 0), dtype=x.dtype, device=x.device)
        full = gather_rows(y, self.R, self.world, self.group) if self.world > 1 else y
        return full.reshape(*shape[:-1], self.R)


def local_gemv_into(rt: dict, x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """This rank's slice of a sharded linear into a caller-owned buffer."""
    return radix_ops.gemv_into(rt, x, None, out)


# ------------------------------------------------- fused NVLink gather --

def exchange_handles(handle: bytes, world: int, group=None) -> list:
    """Every rank's 64-byte IPC handle, index = rank (a collective over
    `group`). A rank that has left, or never calls, makes the others raise
    once the process group's timeout runs out; none of them is left waiting
    on a GPU, as no kernel has been launched yet."""
    import torch.distributed as dist

    handles = [None] * world
    if world > 1:
        dist.all_gather_object(handles, handle, group=group)
    else:
        handles[0] = handle
    return handles


class PeerGather:
    """The gathered outputs of a sequence of row-sharded linears on the GPUs
    of one box: per linear a buffer [M][world * slot] on every rank, which
    every rank's GEMV writes its rows into over NVLink (plain peer stores,
    CUDA IPC mappings; no multicast), and per linear `world` flag words the
    writers raise to their launch count. dm_gemv_gather fuses both into the
    GEMV; linear i may wait for linear `wait` before reading its activations.

    All ranks build it collectively (the IPC handles travel over `group`)
    with the same `slots`; close() (collective) unmaps and frees it."""

    def __init__(self, slots, M: int, out_dtype, rank: int, world: int, device, group=None):
        import ctypes as ct

        from . import _lib

        if not 1 <= world <= _lib.DM_MAX_RANKS:
            raise ValueError(f"PeerGather: world {world} outside 1..{_lib.DM_MAX_RANKS}")
        self.slots = [int(s) for s in slots]
        self.M, self.rank, self.world, self.group = int(M), int(rank), int(world), group
        self.dtype = out_dtype
        self.device = torch.device(device)
        esz = 4 if out_dtype == torch.float32 else 2
        off, at = [], 0
        for s in self.slots:
            off.append(at)
            at += -(-self.M * self.world * s * esz // 256) * 256
        self.flag_off = at  # per linear: world flag words, 64-byte aligned
        at += len(self.slots) * 64 * (-(-self.world * 4 // 64))
        self.cnt_off = at  # per linear: gen, done (this rank's own); then the abort word
        at += len(self.slots) * 8 + 4
        self.out_off, self.bytes = off, -(-at // 256) * 256
        base = ct.c_void_p()
        _lib.call("dm_device_alloc", self.device.index, self.bytes, ct.byref(base))
        self.base = base.value
        h = (ct.c_uint8 * 64)()
        _lib.call("dm_ipc_handle", ct.c_void_p(self.base), h)
        try:
            handles = exchange_handles(bytes(h), self.world, group)
        except Exception:
            _lib.call("dm_device_free", ct.c_void_p(self.base))
            self.base = None
            raise
        self.peer_base = []
        for r in range(self.world):
            if r == self.rank:
                self.peer_base.append(self.base)
                continue
            hp = (ct.c_uint8 * 64).from_buffer_copy(handles[r])
            p = ct.c_void_p()
            _lib.call("dm_ipc_open", hp, self.device.index, ct.byref(p))
            self.peer_base.append(p.value)

    def _flags(self, base: int, i: int) -> int:
        return base + self.flag_off + i * 64 * (-(-self.world * 4 // 64))

    def desc(self, i: int, wait: int | None = None, wait_polls: int = 0):
        """The dm_gather of linear i (waiting for linear `wait` first, giving
        up after `wait_polls` flag polls; 0: the library's bound)."""
        from . import _lib

        g = _lib.Gather()
        g.world, g.rank, g.slot = self.world, self.rank, self.slots[i]
        for r in range(self.world):
            g.peer_out[r] = self.peer_base[r] + self.out_off[i]
            g.peer_flags[r] = self._flags(self.peer_base[r], i)
        g.gen = self.base + self.cnt_off + 8 * i
        g.done = self.base + self.cnt_off + 8 * i + 4
        g.abort = self.base + self.cnt_off + 8 * len(self.slots)
        if wait is not None:
            g.wait_flags = self._flags(self.base, wait)
            g.wait_gen = self.base + self.cnt_off + 8 * wait
        g.wait_polls = int(wait_polls)
        return g

    def launch_count(self, i: int) -> torch.Tensor:
        """This rank's launch count of linear i (a one-element int32 view of
        the device word the flags are compared with)."""
        return device_view(self.base + self.cnt_off + 8 * i, (1,), torch.int32, self.device)

    def abort_word(self) -> torch.Tensor:
        """This rank's abort word (nonzero once a wait has given up)."""
        return device_view(self.base + self.cnt_off + 8 * len(self.slots), (1,), torch.int32, self.device)

    def output(self, i: int) -> torch.Tensor:
        """This rank's gathered output of linear i, [M, world * slot]
        (rank k's rows at [k * slot, k * slot + rows_k))."""
        return device_view(self.base + self.out_off[i], (self.M, self.world * self.slots[i]), self.dtype, self.device)

    def gemv(self, rt: dict, x: torch.Tensor, i: int, wait: int | None = None, bias=None,
             wait_polls: int = 0) -> None:
        """This rank's rows of linear i (runtime dict `rt`), gathered into every
        rank's output(i) and published; the activations `x` [M, C] bf16. A
        wait that gives up is recorded in the tensor's device error word
        (kErrWaitPeer = 4, read by rt["rx_handle"].device_error()) and in the
        abort word, after which every later wait of this rank returns at once."""
        import ctypes as ct

        from . import _lib

        h = rt["rx_handle"]
        if x.dtype != torch.bfloat16 or not x.is_contiguous():
            raise ValueError("PeerGather.gemv: activations must be contiguous bf16")
        b = bias.to(device=x.device, dtype=torch.bfloat16).contiguous() if bias is not None else None
        _lib.call("dm_gemv_gather", h.ptr, ct.c_void_p(x.data_ptr()), x.shape[0],
                  ct.c_void_p(b.data_ptr() if b is not None else 0), _lib.DM_F32 if self.dtype == torch.float32
                  else _lib.DM_BF16, ct.byref(self.desc(i, wait, wait_polls)),
                  ct.c_void_p(torch.cuda.current_stream(x.device).cuda_stream))

    def chain(self, links, wait_polls: int = 0) -> "GatherChain":
        """One persistent launch over a sequence of this gather's linears
        (dm_chain_create): `links` = [(rt, x, i, wait, bias), ...] — linear i
        of this plan computed from activations x (contiguous bf16 [M, C],
        16-byte aligned, e.g. another linear's output(j)[:, :C]), first
        waiting for linear `wait`'s flags (an index into `links`: an earlier
        link's output of this launch, or a later link's of the previous one;
        None: no wait). Same result bits as calling gemv() link by link. The
        plan's flags then belong to the chain: no per-linear gemv() calls.
        A wait gives up after `wait_polls` polls (0: the library's bound),
        recording kErrWaitPeer in the waiting link's tensor and the abort word."""
        import ctypes as ct

        from . import _lib

        arr = (_lib.ChainLink * len(links))()
        keep = []
        for k, (rt, x, i, wait, bias) in enumerate(links):
            if x.dtype != torch.bfloat16 or not x.is_contiguous() or x.shape[0] != self.M:
                raise ValueError(f"PeerGather.chain: link {k}: activations must be contiguous bf16 [M, C]")
            b = bias.to(device=x.device, dtype=torch.bfloat16).contiguous() if bias is not None else None
            keep.append((rt, x, b))
            arr[k].t = rt["rx_handle"].ptr.value
            arr[k].x = x.data_ptr()
            arr[k].bias = b.data_ptr() if b is not None else None
            arr[k].g = self.desc(i, None, wait_polls)
            arr[k].wait = -1 if wait is None else int(wait)
        out = ct.c_void_p()
        _lib.call("dm_chain_create", arr, len(links), self.M,
                  _lib.DM_F32 if self.dtype == torch.float32 else _lib.DM_BF16, ct.byref(out))
        return GatherChain(out.value, self.device, keep)

    def close(self) -> None:
        """Collective: every rank stops using the others' memory, then unmaps."""
        import ctypes as ct

        import torch.distributed as dist

        from . import _lib

        if self.base is None:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)
        for r, p in enumerate(self.peer_base):
            if r != self.rank:
                _lib.call("dm_ipc_close", ct.c_void_p(p))
        _lib.call("dm_device_free", ct.c_void_p(self.base))
        self.base = None


class GatherChain:
    """A chain of row-sharded linears in one persistent launch (dm_chain_run):
    run() enqueues it on the current stream (capturable in a CUDA graph).
    Holds the activations and biases it was built over."""

    def __init__(self, handle: int, device, keep):
        self.handle, self.device, self._keep = handle, device, keep

    def run(self, stream=None) -> None:
        import ctypes as ct

        from . import _lib

        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        _lib.call("dm_chain_run", ct.c_void_p(self.handle), ct.c_void_p(s.cuda_stream))

    def close(self) -> None:
        import ctypes as ct

        from . import _lib

        if self.handle:
            torch.cuda.synchronize(self.device)
            _lib.call("dm_chain_destroy", ct.c_void_p(self.handle))
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
