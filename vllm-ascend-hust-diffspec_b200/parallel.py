"""Head-sharded chunk-score exchange across GPUs.

The reference all-reduces each rank's head-mean chunk scores over the target
TP group and divides by the TP size (diffspec/runtime.py:1292-1297).  The
summation order of an all-reduce depends on the number of ranks, so the
selected chunks could change with the GPU count.  Here every rank computes
the unnormalised mass of each of its kv heads (deterministic, see the score
kernel), the per-kv-head vectors are all-gathered over NCCL, and every rank
sums them in global kv-head order inside the selection kernel, which reads
the all-gather's rank-major layout directly.  The result is bit-identical for
any number of ranks that holds the kv heads in contiguous, rank-ordered
shards.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

__all__ = ["gather_head_scores", "head_major", "shard_heads"]


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
    """All-gather ``[rows, Hk_local, N]`` mass into ``[world, rows, Hk_local, N]``.

    Rank w's slice is its local mass, so global kv head ``w * Hk_local + i``
    is ``result[w, :, i]`` when shards are contiguous and rank-ordered.  The
    selection reads this layout in place (``selection.select_rows`` with a
    4-D ``parts``), so the exchange is the collective alone, with no
    reordering copy.  ``out`` (optional) is the ``[world, rows, Hk_local, N]``
    buffer to gather into; with one rank the result is ``local[None]``.
    """
    world = dist.get_world_size(group)
    rows, hk_local, n = local.shape
    if world == 1:
        return local.unsqueeze(0)
    if out is None:
        out = torch.empty((world, rows, hk_local, n), dtype=local.dtype, device=local.device)
    if out.shape != (world, rows, hk_local, n) or not out.is_contiguous():
        raise ValueError("out must be a contiguous [world, rows, Hk_local, N] buffer")
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, local.contiguous(), group=group)
    else:  # gloo (CPU tests) has no all_gather_into_tensor
        dist.all_gather(list(out.unbind(0)), local.contiguous(), group=group)
    return out


def head_major(gathered: torch.Tensor) -> torch.Tensor:
    """``[world, rows, Hk_local, N]`` -> ``[rows, Hk, N]`` in global kv-head
    order (a copy; the selection does not need it)."""
    world, rows, hk_local, n = gathered.shape
    return gathered.permute(1, 0, 2, 3).reshape(rows, world * hk_local, n)
