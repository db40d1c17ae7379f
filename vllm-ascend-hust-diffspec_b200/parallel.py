"""Head-sharded chunk-score exchange across GPUs.

The reference all-reduces each rank's head-mean chunk scores over the target
TP group and divides by the TP size (diffspec/runtime.py:1292-1297).  The
summation order of an all-reduce depends on the number of ranks, so the
selected chunks could change with the GPU count.  Here every rank computes
the unnormalised mass of each of its kv heads (deterministic, see the score
kernel), the per-kv-head vectors are all-gathered over NCCL, and every rank
sums them in global kv-head order inside the selection kernel.  The result is
bit-identical for any number of ranks that holds the kv heads in contiguous,
rank-ordered shards.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

__all__ = ["gather_head_scores", "shard_heads"]


def shard_heads(num_kv_heads: int, world_size: int, rank: int) -> tuple[int, int]:
    """Contiguous kv-head range ``[start, stop)`` owned by ``rank``."""
    if world_size <= 0 or num_kv_heads % world_size:
        raise ValueError("kv heads must divide evenly across the head-sharding ranks")
    per = num_kv_heads // world_size
    return rank * per, (rank + 1) * per


def gather_head_scores(
    local: torch.Tensor,
    group: dist.ProcessGroup | None = None,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """All-gather ``[rows, Hk_local, N]`` mass into ``[rows, Hk_local * world, N]``.

    The result is ordered by (rank, local kv head), i.e. by global kv head
    when shards are contiguous and rank-ordered.
    """
    world = dist.get_world_size(group)
    if world == 1:
        return local
    rows, hk_local, n = local.shape
    stacked = torch.empty((world, rows, hk_local, n), dtype=local.dtype, device=local.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(stacked, local.contiguous(), group=group)
    else:  # gloo (CPU tests) has no all_gather_into_tensor
        dist.all_gather(list(stacked.unbind(0)), local.contiguous(), group=group)
    if out is None:
        out = torch.empty((rows, world * hk_local, n), dtype=local.dtype, device=local.device)
    out.view(rows, world, hk_local, n).copy_(stacked.permute(1, 0, 2, 3))
    return out
