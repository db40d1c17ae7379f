"""Head-sharded score exchange on two gloo ranks (CPU): the gathered
per-kv-head mass is ordered by global kv head and yields the same selection
as a single rank holding every head."""

from __future__ import annotations

import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import load_package


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys
        sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        from oracle import diffspec_oracle as O

        dsb = load_package()
        rng = np.random.Generator(np.random.PCG64(5))
        rows, hq, hk, d, bs, c, length = 3, 16, 4, 64, 16, 32, 640
        q = O.round_to(rng.standard_normal((rows, hq, d), dtype=np.float32), "bf16")
        kc = O.round_to(rng.standard_normal((rows * length // bs, bs, hk, d), dtype=np.float32), "bf16")
        table = rng.permutation(rows * length // bs).reshape(rows, -1)
        seq = np.array([640, 500, 97])
        lse = rng.random((rows, hq)).astype(np.float32) + 5
        full = O.paged_chunk_head_scores(q, kc, lse, table, seq, c, length, d ** -0.5, acc=np.float32)
        per = hk // world
        heads = slice(rank * per, (rank + 1) * per)
        qh = slice(rank * per * (hq // hk), (rank + 1) * per * (hq // hk))
        local = O.paged_chunk_head_scores(q[:, qh], kc[:, :, heads], lse[:, qh], table, seq, c,
                                          length, d ** -0.5, acc=np.float32)
        gathered = dsb.parallel.gather_head_scores(torch.from_numpy(np.ascontiguousarray(local)))
        # rank-major [world, rows, Hk_local, N], the layout the selection reads
        ok = tuple(gathered.shape) == (world, rows, per, full.shape[-1])
        ok = ok and all(np.array_equal(gathered[w].numpy(), full[:, w * per:(w + 1) * per])
                        for w in range(world))
        ok = ok and np.array_equal(dsb.parallel.head_major(gathered).numpy(), full)
        queue.put((rank, bool(ok), dsb.parallel.shard_heads(hk, world, rank)))
    finally:
        dist.destroy_process_group()


def test_gather_head_scores_two_ranks():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted(queue.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [r[1] for r in results] == [True, True]
    assert [r[2] for r in results] == [(0, 2), (2, 4)]
