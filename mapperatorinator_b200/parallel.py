"""Row sharding across GPUs (one process per GPU, no collective on the path).

Rows of the decode step are independent, so N GPUs split the batch: rank r
owns CFG pairs ``[r*P/N, (r+1)*P/N)`` and keeps both halves of each pair
(rows ``i`` and ``P + i`` of the global ``[2P, V]`` logits), re-packed as a
local ``[cond block; uncond block]``.  torch.distributed is used only for the
plumbing around the step: a barrier before and after the timed region and a
max over ranks of the device time.
"""

from __future__ import annotations

import torch


def shard_range(total: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [start, end) of `total` rows for `rank` (sizes differ by <= 1)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def local_cfg_rows(logits: torch.Tensor, pairs: int, start: int, end: int) -> torch.Tensor:
    """This rank's [2n, V] block of a global [2P, V] CFG logits matrix:
    first-half rows start..end-1 followed by their partners P+start..P+end-1."""
    if logits.shape[0] != 2 * pairs:
        raise ValueError("expected [2 * pairs, V] logits")
    return torch.cat([logits[start:end], logits[pairs + start:pairs + end]], dim=0)


def max_over_ranks(value: float, device=None) -> float:
    """Max of a scalar over every rank of the default process group (identity
    without one)."""
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
