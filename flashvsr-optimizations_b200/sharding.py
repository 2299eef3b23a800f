"""Token-row sharding of the FFN across ranks (one process per GPU).

Token rows are independent through the whole FFN, so the path partitions them:
each rank runs the FFN on a contiguous block of rows with replicated weights,
and no collective sits inside a layer.  Outputs are gathered with one
all-gather (NCCL over NVLink on GPUs, gloo in the CPU tests) when a single
rank needs all of them.  Global scales are per shard: each shard computes
exactly what the reference computes when run on that shard.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

__all__ = ["row_range", "shard_rows", "gather_rows", "ShardedFFN"]


def row_range(total: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of `rank`'s contiguous block; the first total % world ranks get one more row."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    if total < 0:
        raise ValueError("total must be >= 0")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_rows(x: torch.Tensor, world: int, rank: int) -> torch.Tensor:
    """This rank's rows of a [tokens, ...] tensor (a view)."""
    start, stop = row_range(x.shape[0], world, rank)
    return x[start:stop]


def gather_rows(local: torch.Tensor, total: int, group=None) -> torch.Tensor:
    """All-gather row blocks made by `row_range` back into the full [total, ...] tensor.

    Blocks may differ by one row; each is padded to the largest block for the
    fixed-size collective and the padding is dropped afterwards.
    """
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    start, stop = row_range(total, world, rank)
    if local.shape[0] != stop - start:
        raise ValueError(f"rank {rank}: expected {stop - start} rows, got {local.shape[0]}")
    biggest = row_range(total, world, 0)[1]
    padded = local.new_zeros((biggest, *local.shape[1:]))
    padded[: local.shape[0]] = local
    out = local.new_empty((world * biggest, *local.shape[1:]))
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, padded.contiguous(), group=group)
    else:
        dist.all_gather(list(out.chunk(world)), padded.contiguous(), group=group)
    parts = []
    for r in range(world):
        s, e = row_range(total, world, r)
        parts.append(out[r * biggest: r * biggest + (e - s)])
    return torch.cat(parts, dim=0)


class ShardedFFN(torch.nn.Module):
    """Run `ffn` on this rank's token rows and all-gather the result.

    `forward(x)` takes the full [tokens, d] activation (every rank holds it, as
    when a video chunk is broadcast) and returns the full output on every rank.
    """

    def __init__(self, ffn: torch.nn.Module, group=None):
        super().__init__()
        self.ffn = ffn
        self.group = group

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        world = dist.get_world_size(self.group)
        rank = dist.get_rank(self.group)
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        local = shard_rows(x2, world, rank)
        y_local = self.ffn(local) if local.shape[0] > 0 else local.new_empty((0, shape[-1]))
        y = gather_rows(y_local, x2.shape[0], self.group)
        return y.reshape(*shape[:-1], y.shape[-1])
