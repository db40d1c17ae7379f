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

import ctypes

import torch
import torch.distributed as dist

from . import _lib

__all__ = ["PeerExchange", "gather_head_scores", "head_major", "peer_all_gather", "shard_heads"]


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


def peer_all_gather(local: torch.Tensor, site: "PeerExchange", out: torch.Tensor) -> torch.Tensor:
    """All-gather of fp32 ``local`` over NVLink peer memory into ``out``
    (``[world, *local.shape]``, rank-major, as ``all_gather_into_tensor``
    writes it): this rank's values, tagged with the call's number, are stored
    into every rank's buffer of ``site`` (``PeerExchange.create(1, count,
    ...)``, count = ``local.numel()`` rounded up to 8 or more), then each rank
    unpacks its own buffer once the tags show every rank's values arrived
    (``dsb_peer_all_gather_send`` / ``_recv``, two launches, no collective)."""
    n = local.numel()
    if local.dtype != torch.float32 or not local.is_contiguous() or n % 8 or n > site.features:
        raise ValueError("local must be contiguous fp32 with a multiple of 8 elements that fit the site")
    if out.dtype != torch.float32 or not out.is_contiguous() or out.numel() != site.world * n:
        raise ValueError("out must be contiguous fp32 [world, *local.shape]")
    device = _lib.require_cuda(local, out)
    stream = _lib.stream_ptr(device)
    _lib.call("dsb_peer_all_gather_send", _lib.ptr(local), n, _lib.ptr(site.bases), site.world,
              site.rank, site.features, site.own_base, stream)
    _lib.call("dsb_peer_all_gather_recv", site.own_base, site.world, n, site.features,
              _lib.ptr(out), _lib.ptr(_lib.error_flag(device)), stream)
    return out


def head_major(gathered: torch.Tensor) -> torch.Tensor:
    """``[world, rows, Hk_local, N]`` -> ``[rows, Hk, N]`` in global kv-head
    order (a copy; the selection does not need it)."""
    world, rows, hk_local, n = gathered.shape
    return gathered.permute(1, 0, 2, 3).reshape(rows, world * hk_local, n)


class PeerExchange:
    """One all-reduce site of the fused row-split linear + all-reduce
    (``dsb_draft_linear_peer`` then ``dsb_peer_add_rms_norm``): this rank's
    exchange buffer and every rank's buffer as mapped in this process.

    :meth:`create` (collective over ``group``) allocates the buffer through
    the library, sends its CUDA IPC handle to the other ranks
    (``all_gather_object``, any backend) and maps theirs: plain peer mappings
    over NVLink, no multicast.  :meth:`local` builds ``world`` virtual ranks
    whose buffers all live on one GPU, so the exchange's layout and sums can
    be run rank after rank on a single device.  Every rank must then issue
    the same sequence of calls on the site; the call count lives in the
    buffers, so the sequence can be captured in a CUDA graph.  :meth:`close`
    unmaps and frees."""

    def __init__(self, world: int, rank: int, tokens_max: int, features: int,
                 device: torch.device, own_base: int, bases: list[int], owned: bool,
                 opened: list[int]):
        self.world, self.rank = world, rank
        self.tokens_max, self.features = tokens_max, features
        self.device = device
        self.own_base = own_base
        self.bases = torch.tensor(bases, dtype=torch.int64, device=device)
        self._owned, self._opened = owned, opened

    @staticmethod
    def _alloc(world, tokens_max, features) -> int:
        base = ctypes.c_void_p()
        _lib.call("dsb_peer_buffer_create", world, tokens_max, features, ctypes.byref(base))
        return int(base.value)

    @classmethod
    def create(cls, tokens_max: int, features: int, device: torch.device,
               group: dist.ProcessGroup | None = None) -> "PeerExchange":
        world, rank = dist.get_world_size(group), dist.get_rank(group)
        with torch.cuda.device(device):
            own = cls._alloc(world, tokens_max, features)
            handle = ctypes.create_string_buffer(64)
            _lib.call("dsb_ipc_handle", ctypes.c_void_p(own), handle)
            handles = [None] * world
            dist.all_gather_object(handles, bytes(handle.raw), group=group)
            bases, opened = [], []
            for q in range(world):
                if q == rank:
                    bases.append(own)
                    continue
                peer = ctypes.c_void_p()
                _lib.call("dsb_ipc_open", ctypes.create_string_buffer(handles[q], 64),
                          ctypes.byref(peer))
                bases.append(int(peer.value))
                opened.append(int(peer.value))
        return cls(world, rank, tokens_max, features, device, own, bases, True, opened)

    @classmethod
    def local(cls, world: int, tokens_max: int, features: int,
              device: torch.device) -> list["PeerExchange"]:
        with torch.cuda.device(device):
            bases = [cls._alloc(world, tokens_max, features) for _ in range(world)]
        sites = [cls(world, r, tokens_max, features, device, bases[r], bases, False, [])
                 for r in range(world)]
        sites[0]._local_all = bases  # rank 0 frees every virtual rank's buffer
        return sites

    def close(self) -> None:
        with torch.cuda.device(self.device):
            for base in self._opened:
                _lib.call("dsb_ipc_close", ctypes.c_void_p(base))
            self._opened = []
            if self._owned:
                _lib.call("dsb_peer_buffer_destroy", ctypes.c_void_p(self.own_base))
                self._owned = False
            for base in getattr(self, "_local_all", []):
                _lib.call("dsb_peer_buffer_destroy", ctypes.c_void_p(base))
            self._local_all = []
