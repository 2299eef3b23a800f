"""Token-row sharding of the FFN across ranks (one process per GPU).

Token rows are independent through the whole FFN, so the path partitions them:
each rank runs the FFN on a contiguous block of rows with replicated weights,
and no collective sits inside a layer.  Outputs are gathered with one
all-gather (NCCL over NVLink on GPUs, gloo in the CPU tests) when a single
rank needs all of them.  By default global scales are per shard: each shard
computes exactly what the reference computes when run on that shard.  With
``global_scales=True`` an NVFP4 FFN instead all-reduces (MAX) the 4-byte amax
of each activation it quantizes -- x, then the GELU output h -- so every shard
uses the scale of the whole tensor and the gathered output equals the
single-GPU result bit for bit (two tiny collectives per layer; off by
default).  The FP8 mode's scales are per row, so its shards agree with the
single-GPU result either way.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

__all__ = ["row_range", "shard_rows", "gather_rows", "global_amax", "nvfp4_ffn_global_scales",
           "ShardedFFN"]


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


def gather_rows(local: torch.Tensor, total: int, group=None,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """All-gather row blocks made by `row_range` back into the full [total, ...] tensor.

    When every rank holds the same number of rows (total % world == 0, as for the stack
    workloads on 1/2/4/8 GPUs) the blocks are gathered straight into `out` with one
    all_gather_into_tensor: no padding, no concatenation.  Uneven blocks (they differ by
    one row) are padded to the largest block for the fixed-size collective, and the
    ranks after the first total % world are moved down by their missing rows afterwards.
    `out` (optional) receives the result and is returned.
    """
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    start, stop = row_range(total, world, rank)
    if local.shape[0] != stop - start:
        raise ValueError(f"rank {rank}: expected {stop - start} rows, got {local.shape[0]}")
    shape = (total, *local.shape[1:])
    if out is None:
        out = local.new_empty(shape)
    elif tuple(out.shape) != shape or out.dtype != local.dtype or not out.is_contiguous():
        raise ValueError(f"out must be a contiguous {local.dtype} tensor of shape {shape}")
    nccl = dist.get_backend(group) == "nccl"
    base, extra = divmod(total, world)
    local = local.contiguous()
    if extra == 0:
        if nccl:
            dist.all_gather_into_tensor(out, local, group=group)
        else:
            dist.all_gather(list(out.chunk(world)), local, group=group)
        return out
    biggest = base + 1
    padded = local.new_empty((biggest, *local.shape[1:]))
    padded[: local.shape[0]] = local
    if local.shape[0] < biggest:
        padded[local.shape[0]:].zero_()
    gathered = local.new_empty((world * biggest, *local.shape[1:]))
    if nccl:
        dist.all_gather_into_tensor(gathered, padded, group=group)
    else:
        dist.all_gather(list(gathered.chunk(world)), padded, group=group)
    # ranks 0..extra-1 hold `biggest` rows and already sit at their final offsets
    out[: extra * biggest] = gathered[: extra * biggest]
    if world > extra:
        tail = gathered[extra * biggest:].reshape(world - extra, biggest, *local.shape[1:])
        out[extra * biggest:] = tail[:, :base].reshape(-1, *local.shape[1:])
    return out


def global_amax(amax: torch.Tensor, group=None) -> torch.Tensor:
    """max over ranks of a per-rank amax (1-element fp32 tensor), in place; 4 bytes on the wire."""
    dist.all_reduce(amax, op=dist.ReduceOp.MAX, group=group)
    return amax


def nvfp4_ffn_global_scales(x: torch.Tensor, ffn, group=None,
                            reduce_amax=global_amax) -> torch.Tensor:
    """An NVFP4 FFN (NVFP4FFN or Sequential of QuantLinear, GELU, QuantLinear) on this
    rank's rows with the global scales of the whole activation: amax(x) and amax(h) are
    reduced over the ranks before each quantization (ffn_quantization.py:29-32 applied to
    the full tensor).  `reduce_amax(amax, group)` is the reduction (all_reduce MAX)."""
    from . import ops
    l1, l2 = ffn[0], ffn[2]
    a = ops.amax(x) if x.shape[0] > 0 else x.new_zeros(1, dtype=torch.float32)
    a = reduce_amax(a, group)
    if x.shape[0] == 0:  # this rank has no rows: it still takes part in both reductions
        reduce_amax(x.new_zeros(1, dtype=torch.float32), group)
        return x.new_empty((0, l2.out_features))
    q, s, g = ops.nvfp4_quantize_from_amax(x, a)
    h, amax_h = ops.nvfp4_gemm(q, s, g, l1.qweight, l1.scale, l1.global_sf, l1.bias, gelu=True)
    amax_h = reduce_amax(amax_h, group)
    qh, sh, gh = ops.nvfp4_quantize_from_amax(h, amax_h)
    y, _ = ops.nvfp4_gemm(qh, sh, gh, l2.qweight, l2.scale, l2.global_sf, l2.bias, gelu=False)
    return y


class ShardedFFN(torch.nn.Module):
    """Run `ffn` on this rank's token rows and all-gather the result.

    `forward(x)` takes the full [tokens, d] activation (every rank holds it, as
    when a video chunk is broadcast) and returns the full output on every rank.
    `global_scales=True` (NVFP4 FFNs): scales of the whole tensor, see
    nvfp4_ffn_global_scales.
    """

    def __init__(self, ffn: torch.nn.Module, group=None, global_scales: bool = False):
        super().__init__()
        self.ffn = ffn
        self.group = group
        self.global_scales = global_scales

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        world = dist.get_world_size(self.group)
        rank = dist.get_rank(self.group)
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        local = shard_rows(x2, world, rank)
        if self.global_scales:
            y_local = nvfp4_ffn_global_scales(local, self.ffn, self.group)
        else:
            y_local = self.ffn(local) if local.shape[0] > 0 else local.new_empty((0, shape[-1]))
        y = gather_rows(y_local, x2.shape[0], self.group)
        return y.reshape(*shape[:-1], y.shape[-1])
