"""Tensor-parallel Eagle3 draft layer (Eagle3DraftLayerTP) at config 5's shape
against the single-GPU layer, on one GPU: every shard of a world size runs
on its own slice of the caches, and the all-reduces are a rank-ordered fp32
sum of the shards' partials (what NCCL's sum computes up to order).  World 1
is bit-identical to Eagle3DraftLayer.step (output and cache rows); worlds 2,
4 and 8 (8: kv heads replicated on two ranks each) meet the path's bf16
tolerance in the output and in the raw / working-cache rows of their kv
heads."""

from __future__ import annotations

import pytest
import torch

from conftest import close_bf16

pytestmark = pytest.mark.gpu

HIDDEN, QKV_IN, HQ, HK, D, INTER, N, SLOTS, MAX_LEN, BUDGET = (
    2048, 4096, 32, 4, 128, 6144, 16, 16, 4096, 2048)


def _inputs(cuda):
    g = torch.Generator(device="cpu").manual_seed(21)
    bf = torch.bfloat16
    dev = lambda t: t.to(cuda)  # noqa: E731
    inv = 1.0 / (1e6 ** (torch.arange(0, D, 2, dtype=torch.float64) / D))
    fr = torch.arange(BUDGET, dtype=torch.float64)[:, None] * inv[None]
    return dict(
        x_in=dev(torch.randn((N, QKV_IN), generator=g)).to(bf),
        residual=dev(torch.randn((N, HIDDEN), generator=g)).to(bf),
        slots=dev(torch.randperm(SLOTS, generator=g)[:N].to(torch.int32)),
        abs_pos=dev(torch.randint(BUDGET, MAX_LEN, (N,), generator=g)),
        local_pos=dev(torch.randint(2, BUDGET - 4, (N,), generator=g).to(torch.int32)),
        wk=dev(torch.randn((SLOTS, HK, BUDGET, D), generator=g)).to(bf),
        wv=dev(torch.randn((SLOTS, HK, BUDGET, D), generator=g)).to(bf),
        cos_sin=dev(torch.cat((fr.cos(), fr.sin()), -1)).to(bf))


def _run_full(layer, inp, offset, cuda):
    raw_k = torch.zeros((SLOTS, MAX_LEN, HK, D), dtype=torch.bfloat16, device=cuda)
    raw_v = torch.zeros_like(raw_k)
    wk, wv = inp["wk"].clone(), inp["wv"].clone()
    out = layer.step(inp["x_in"], inp["residual"], slots=inp["slots"], abs_positions=inp["abs_pos"],
                     local_positions=inp["local_pos"] - offset, position_offset=offset,
                     raw_key=raw_k, raw_value=raw_v, working_key=wk, working_value=wv,
                     cos_sin=inp["cos_sin"])
    return out, raw_k, raw_v, wk, wv


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_tp_shards_match_single_gpu_layer(dsb, cuda, world):
    dl = dsb.draft_layer
    full = dl.Eagle3DraftLayer(cuda, seed=9)
    inp = _inputs(cuda)
    offset = 1
    ref, raw_k, raw_v, wk_ref, wv_ref = _run_full(full, inp, offset, cuda)
    shards = [dl.Eagle3DraftLayerTP(full, r, world, all_reduce=lambda t: None) for r in range(world)]
    caches = []
    for sh in shards:
        heads = sh.kv_heads
        caches.append(dict(
            raw_k=torch.zeros((SLOTS, MAX_LEN, sh.hk, D), dtype=torch.bfloat16, device=cuda),
            raw_v=torch.zeros((SLOTS, MAX_LEN, sh.hk, D), dtype=torch.bfloat16, device=cuda),
            wk=inp["wk"][:, heads].contiguous(), wv=inp["wv"][:, heads].contiguous()))
    kw = dict(slots=inp["slots"], abs_positions=inp["abs_pos"],
              local_positions=inp["local_pos"] - offset, position_offset=offset,
              cos_sin=inp["cos_sin"])
    parts = [sh.attention_partial(inp["x_in"], raw_key=c["raw_k"], raw_value=c["raw_v"],
                                  working_key=c["wk"], working_value=c["wv"], **kw)
             for sh, c in zip(shards, caches)]
    o_sum = parts[0].clone()
    for p in parts[1:]:
        o_sum += p  # rank order, fp32
    mlp = [sh.mlp_partial(o_sum, inp["residual"]) for sh in shards]
    d_sum = mlp[0][1].clone()
    for _, p in mlp[1:]:
        d_sum += p
    outs = [sh.finish(d_sum, x) for sh, (x, _) in zip(shards, mlp)]
    torch.cuda.synchronize()
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0
    for o in outs[1:]:
        assert torch.equal(o, outs[0])  # every rank holds the same layer output
    if world == 1:
        assert torch.equal(outs[0], ref)
    else:
        close_bf16(outs[0].float().cpu().numpy(), ref.float().cpu().numpy())
    # this rank's kv heads: the single-GPU layer's cache rows (bit for bit at
    # world 1; with fewer weight tiles a shard's projection splits K
    # differently, so beyond world 1 the fp32 sums round within the tolerance)
    slots, pos = inp["slots"].long(), inp["abs_pos"].long()
    for sh, c in zip(shards, caches):
        h = sh.kv_heads
        for mine, ref_cache in ((c["raw_k"], raw_k), (c["raw_v"], raw_v)):
            got, want = mine[slots, pos], ref_cache[slots, pos][:, h]
            if world == 1:
                assert torch.equal(mine, ref_cache)
            else:
                close_bf16(got.float().cpu().numpy(), want.float().cpu().numpy())
        for mine, ref_cache in ((c["wk"], wk_ref), (c["wv"], wv_ref)):
            if world == 1:
                assert torch.equal(mine, ref_cache)
            else:
                close_bf16(mine.float().cpu().numpy(), ref_cache[:, h].float().cpu().numpy())


def test_add_rms_norm_matches_separate_ops(dsb, cuda):
    """dsb_add_rms_norm: round(partial + residual) and then dsb_rms_norm's
    output bit for bit, with and without the norm."""
    dl = dsb.draft_layer
    g = torch.Generator(device=cuda).manual_seed(3)
    for rows, cols in ((16, 2048), (5, 4096), (1, 8)):
        p = torch.randn((rows, cols), generator=g, device=cuda) * 3
        r = torch.randn((rows, cols), generator=g, device=cuda).bfloat16()
        w = (torch.rand((cols,), generator=g, device=cuda) + 0.5).bfloat16()
        x, normed = dl.add_rms_norm(p, r, w, 1e-6)
        assert torch.equal(x, (p + r.float()).bfloat16())
        assert torch.equal(normed, dl.rms_norm(x, w, 1e-6))
        x2, none = dl.add_rms_norm(p, r, None, 1e-6)
        assert none is None and torch.equal(x2, x)
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0
