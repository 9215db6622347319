"""Box sharding across ranks and the gather of final bounds.

Bounding is independent per input box (Luna bounds one box per
TorchModel::compute_bounds call), so a batch partitions into contiguous
ranges, one per rank, with no exchange while bounding; the only collective
is the gather of the final [boxes, nspec] lower/upper bounds at the end.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def shard_range(rank: int, world: int, n: int) -> tuple[int, int]:
    """Contiguous [begin, end) of n boxes for `rank`; sizes differ by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    base, extra = divmod(n, world)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)


def gather_bounds(lb: torch.Tensor, ub: torch.Tensor, counts: list[int]) -> tuple[torch.Tensor, torch.Tensor]:
    """All-gather each rank's [n_r, nspec] bounds into [sum n_r, nspec] on every
    rank, in rank order.  Uses NCCL for CUDA tensors, any backend otherwise.
    Ranks may hold different box counts (`counts[r]` for rank r)."""
    world = dist.get_world_size()
    nspec = lb.shape[1]
    width = max(counts)
    both = torch.zeros((2, width, nspec), dtype=lb.dtype, device=lb.device)
    both[0, : lb.shape[0]] = lb
    both[1, : ub.shape[0]] = ub
    out = [torch.empty_like(both) for _ in range(world)]
    dist.all_gather(out, both)
    glb = torch.cat([o[0, : counts[r]] for r, o in enumerate(out)])
    gub = torch.cat([o[1, : counts[r]] for r, o in enumerate(out)])
    return glb, gub
