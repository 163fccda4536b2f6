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
