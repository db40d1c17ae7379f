"""Fused row-split linear + all-reduce over peer memory (dsb_draft_linear_peer,
dsb_peer_add_rms_norm), run on one GPU with virtual ranks whose exchange
buffers all live on it (PeerExchange.local): every rank's linear runs before
any rank's add + RMSNorm, so no kernel waits for one that has not been
launched.  Each rank's result must equal, bit for bit, the rank-ordered fp32
sum of the ranks' "partial" linears followed by dsb_add_rms_norm, over
several calls in a row (both buffer parities, ragged token counts); the
tensor-parallel layer's fused stages must equal its all-reduce stages."""

from __future__ import annotations

import pytest
import torch

from test_gpu_draft_layer_tp import D, HK, MAX_LEN, SLOTS, _inputs

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world", [1, 2, 4, 8])
@pytest.mark.parametrize("packed", [False, True])
def test_peer_linear_and_norm_match_rank_ordered_sum(dsb, cuda, world, packed):
    dl = dsb.draft_layer
    features, k, tmax = 2048, 1024, 16
    g = torch.Generator(device=cuda).manual_seed(world * 10 + packed)
    ws = [(torch.randn((features, k), generator=g, device=cuda) / k ** 0.5).bfloat16()
          for _ in range(world)]
    wl = [dl.pack_linear_weight(w) if packed else w for w in ws]
    norm_w = (torch.rand((features,), generator=g, device=cuda) + 0.5).bfloat16()
    sites = dsb.parallel.PeerExchange.local(world, tmax, features, cuda)
    try:
        for call, tokens in enumerate((16, 16, 5, 16)):  # parities 0, 1, 0, 1
            xs = [torch.randn((tokens, k), generator=g, device=cuda).bfloat16() for _ in range(world)]
            res = torch.randn((tokens, features), generator=g, device=cuda).bfloat16()
            parts = [dl.draft_linear(x, w, "partial", packed=packed) for x, w in zip(xs, wl)]
            total = parts[0].clone()
            for p in parts[1:]:
                total += p  # rank order, fp32
            want_x, want_n = dl.add_rms_norm(total, res, norm_w, 1e-6)
            for x, w, site in zip(xs, wl, sites):
                dl.draft_linear_peer(x, w, site, packed=packed)
            for site in sites:
                got_x, got_n = dl.peer_add_rms_norm(site, res, norm_w if call % 2 == 0 else None,
                                                    1e-6)
                assert torch.equal(got_x, want_x), (call, site.rank)
                if call % 2 == 0:
                    assert torch.equal(got_n, want_n), (call, site.rank)
            torch.cuda.synchronize()
            assert dsb._lib.read_and_clear_error_flag(cuda) == 0
    finally:
        sites[0].close()


@pytest.mark.parametrize("world", [1, 2, 8])
def test_tp_layer_peer_stages_match_all_reduce_stages(dsb, cuda, world):
    """Eagle3DraftLayerTP with peer sites: its three fused stages, run rank
    after rank, against its all-reduce stages with a rank-ordered sum, twice
    in a row; world 1 also against the single-GPU layer."""
    dl = dsb.draft_layer
    full = dl.Eagle3DraftLayer(cuda, seed=9)
    inp = _inputs(cuda)
    offset = 1
    o_sites = dsb.parallel.PeerExchange.local(world, 16, full.w_o.shape[0], cuda)
    d_sites = dsb.parallel.PeerExchange.local(world, 16, full.w_o.shape[0], cuda)
    try:
        shards = [dl.Eagle3DraftLayerTP(full, r, world, all_reduce=lambda t: None,
                                        peer=(o_sites[r], d_sites[r])) for r in range(world)]

        def caches():
            return [dict(raw_k=torch.zeros((SLOTS, MAX_LEN, sh.hk, D), dtype=torch.bfloat16,
                                           device=cuda),
                         raw_v=torch.zeros((SLOTS, MAX_LEN, sh.hk, D), dtype=torch.bfloat16,
                                           device=cuda),
                         wk=inp["wk"][:, sh.kv_heads].contiguous(),
                         wv=inp["wv"][:, sh.kv_heads].contiguous()) for sh in shards]

        kw = dict(slots=inp["slots"], abs_positions=inp["abs_pos"],
                  local_positions=inp["local_pos"] - offset, position_offset=offset,
                  cos_sin=inp["cos_sin"])
        for _ in range(2):
            ca, cb = caches(), caches()
            parts = [sh.attention_partial(inp["x_in"], raw_key=c["raw_k"], raw_value=c["raw_v"],
                                          working_key=c["wk"], working_value=c["wv"], **kw)
                     for sh, c in zip(shards, ca)]
            o_sum = parts[0].clone()
            for p in parts[1:]:
                o_sum += p
            mlp = [sh.mlp_partial(o_sum, inp["residual"]) for sh in shards]
            d_sum = mlp[0][1].clone()
            for _, p in mlp[1:]:
                d_sum += p
            want = [sh.finish(d_sum, x) for sh, (x, _) in zip(shards, mlp)]
            for sh, c in zip(shards, cb):
                sh.attention_peer(inp["x_in"], raw_key=c["raw_k"], raw_value=c["raw_v"],
                                  working_key=c["wk"], working_value=c["wv"], **kw)
            xs = [sh.mlp_peer(inp["residual"]) for sh in shards]
            got = [sh.finish_peer(x) for sh, x in zip(shards, xs)]
            torch.cuda.synchronize()
            assert dsb._lib.read_and_clear_error_flag(cuda) == 0
            for a, b in zip(got, want):
                assert torch.equal(a, b)
            for a, b in zip(cb, ca):
                for key in a:
                    assert torch.equal(a[key], b[key])
        if world == 1:
            raw_k = torch.zeros((SLOTS, MAX_LEN, HK, D), dtype=torch.bfloat16, device=cuda)
            ref = full.step(inp["x_in"], inp["residual"], raw_key=raw_k,
                            raw_value=torch.zeros_like(raw_k), working_key=inp["wk"].clone(),
                            working_value=inp["wv"].clone(), **kw)
            out = shards[0].step(inp["x_in"], inp["residual"], raw_key=raw_k.clone(),
                                 raw_value=torch.zeros_like(raw_k),
                                 working_key=inp["wk"].clone(), working_value=inp["wv"].clone(),
                                 **kw)
            assert torch.equal(out, ref)
    finally:
        o_sites[0].close()
        d_sites[0].close()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_peer_all_gather_matches_stack(dsb, cuda, world):
    """peer_all_gather with virtual ranks on one GPU (every send before any
    receive): each rank's out is the rank-major stack of every rank's local
    block, bit for bit, over three calls (both parities, a shorter count) and
    at the retrieval's shape ([rows, Hk_local, chunks])."""
    rows, hk_local, chunks = 32, 2, 640
    count = rows * hk_local * chunks
    g = torch.Generator(device=cuda).manual_seed(world)
    sites = dsb.parallel.PeerExchange.local(world, 1, count, cuda)
    try:
        for call, shape in enumerate(((rows, hk_local, chunks), (rows, hk_local, chunks),
                                      (rows // 2, hk_local, chunks))):
            local = [torch.rand(shape, generator=g, device=cuda) for _ in range(world)]
            outs = [torch.full((world, *shape), float("nan"), device=cuda) for _ in range(world)]
            for r, site in enumerate(sites):
                dsb._lib.call("dsb_peer_all_gather_send", local[r].data_ptr(), local[r].numel(),
                              site.bases.data_ptr(), world, r, site.features, site.own_base,
                              dsb._lib.stream_ptr(cuda))
            for r, site in enumerate(sites):
                dsb._lib.call("dsb_peer_all_gather_recv", site.own_base, world, local[r].numel(),
                              site.features, outs[r].data_ptr(),
                              dsb._lib.error_flag(cuda).data_ptr(), dsb._lib.stream_ptr(cuda))
            want = torch.stack(local)
            torch.cuda.synchronize()
            assert dsb._lib.read_and_clear_error_flag(cuda) == 0
            for out in outs:
                assert torch.equal(out, want), call
    finally:
        sites[0].close()


def test_peer_waits_run_out_flag_and_finish(dsb, cuda):
    """A rank whose peer never sends: the consumer's bounded waits (2 s) run
    out, the kernels finish with DSB_FLAG_TIMEOUT in the error word, and the
    context stays usable (a normal call afterwards is exact)."""
    dl = dsb.draft_layer
    timeout_bit = 32
    features, k = 256, 128
    g = torch.Generator(device=cuda).manual_seed(5)
    w = (torch.randn((features, k), generator=g, device=cuda) / k ** 0.5).bfloat16()
    x = torch.randn((16, k), generator=g, device=cuda).bfloat16()
    res = torch.randn((16, features), generator=g, device=cuda).bfloat16()
    sites = dsb.parallel.PeerExchange.local(2, 16, features, cuda)
    gsites = dsb.parallel.PeerExchange.local(2, 1, 64, cuda)
    try:
        dl.draft_linear_peer(x, w, sites[0])        # rank 1 never sends
        dl.peer_add_rms_norm(sites[0], res, None, 1e-6)
        torch.cuda.synchronize()
        assert dsb._lib.read_and_clear_error_flag(cuda) & timeout_bit
        local = torch.rand((64,), generator=g, device=cuda)
        out = torch.empty((2, 64), device=cuda)
        dsb._lib.call("dsb_peer_all_gather_send", local.data_ptr(), 64, gsites[0].bases.data_ptr(),
                      2, 0, 64, gsites[0].own_base, dsb._lib.stream_ptr(cuda))
        dsb._lib.call("dsb_peer_all_gather_recv", gsites[0].own_base, 2, 64, 64, out.data_ptr(),
                      dsb._lib.error_flag(cuda).data_ptr(), dsb._lib.stream_ptr(cuda))
        torch.cuda.synchronize()
        assert dsb._lib.read_and_clear_error_flag(cuda) & timeout_bit
        assert torch.equal(out[0], local)  # the slot that did arrive
    finally:
        sites[0].close()
        gsites[0].close()
    part = dl.draft_linear(x, w, "partial")
    got, _ = dl.add_rms_norm(part, res, None, 1e-6)
    assert torch.equal(got, (part + res.float()).bfloat16())
    torch.cuda.synchronize()
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0
