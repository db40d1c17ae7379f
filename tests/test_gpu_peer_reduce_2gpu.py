"""The fused row-split linear + all-reduce across two GPUs, one process each
(skipped with fewer than two GPUs): exchange buffers mapped with CUDA IPC,
partials stored over NVLink, flags waited on across devices.  Every rank's
tensor-parallel layer step (Eagle3DraftLayerTP with peer sites) must equal,
bit for bit, the same layer computed on that rank alone from both shards
with a rank-ordered fp32 sum, over two steps in a row; the peer all-gather
must equal gloo's all_gather of the same blocks, twice.  The handles travel
over a gloo group on 127.0.0.1."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, queue):
    import sys
    from datetime import timedelta

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    ok, msg = False, ""
    try:
        from conftest import load_package
        from test_gpu_draft_layer_tp import D, MAX_LEN, SLOTS, _inputs

        dsb = load_package()
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dl = dsb.draft_layer
        full = dl.Eagle3DraftLayer(dev, seed=9)
        inp = _inputs(dev)
        offset = 1
        kw = dict(slots=inp["slots"], abs_positions=inp["abs_pos"],
                  local_positions=inp["local_pos"] - offset, position_offset=offset,
                  cos_sin=inp["cos_sin"])
        shards = [dl.Eagle3DraftLayerTP(full, r, world, all_reduce=lambda t: None)
                  for r in range(world)]

        def cache(sh):
            return dict(raw_key=torch.zeros((SLOTS, MAX_LEN, sh.hk, D), dtype=torch.bfloat16,
                                            device=dev),
                        raw_value=torch.zeros((SLOTS, MAX_LEN, sh.hk, D), dtype=torch.bfloat16,
                                              device=dev),
                        working_key=inp["wk"][:, sh.kv_heads].contiguous(),
                        working_value=inp["wv"][:, sh.kv_heads].contiguous())

        parts = [sh.attention_partial(inp["x_in"], **cache(sh), **kw) for sh in shards]
        o_sum = parts[0].clone()
        for p in parts[1:]:
            o_sum += p
        mlp = [sh.mlp_partial(o_sum, inp["residual"]) for sh in shards]
        d_sum = mlp[0][1].clone()
        for _, p in mlp[1:]:
            d_sum += p
        want = shards[rank].finish(d_sum, mlp[rank][0])

        hidden = full.w_o.shape[0]
        sites = tuple(dsb.parallel.PeerExchange.create(16, hidden, dev) for _ in range(2))
        dist.barrier()  # both ranks' buffers are mapped before the first call
        mine = dl.Eagle3DraftLayerTP(full, rank, world, peer=sites)
        outs = [mine.step(inp["x_in"], inp["residual"], **cache(mine), **kw) for _ in range(2)]
        torch.cuda.synchronize(dev)
        flag = dsb._lib.read_and_clear_error_flag(dev)
        ok = flag == 0 and all(torch.equal(o, want) for o in outs)
        msg = f"flag {flag}, max diff {max((o.float() - want.float()).abs().max().item() for o in outs)}"
        # the retrieval's all-gather of per-kv-head mass, twice
        gsite = dsb.parallel.PeerExchange.create(1, 16 * 2 * 640, dev)
        dist.barrier()
        for call in range(2):
            mass = torch.rand((16, 2, 640), generator=torch.Generator(device=dev).manual_seed(
                10 * call + rank), device=dev)
            got = dsb.parallel.peer_all_gather(mass, gsite, torch.empty((2, 16, 2, 640), device=dev))
            every = [torch.empty_like(mass).cpu() for _ in range(world)]
            dist.all_gather(every, mass.cpu())
            torch.cuda.synchronize(dev)
            ok = ok and torch.equal(got.cpu(), torch.stack(every))
        ok = ok and dsb._lib.read_and_clear_error_flag(dev) == 0
        dist.barrier()
        gsite.close()
        dist.barrier()  # no rank still writes into the other's buffers
        for site in sites:
            site.close()
        dist.barrier()
    except Exception as error:  # reported to the parent
        msg = repr(error)
    finally:
        queue.put((rank, ok, msg))
        dist.destroy_process_group()


def test_peer_all_reduce_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted(queue.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert [r[1] for r in results] == [True, True], results
