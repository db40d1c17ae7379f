"""The torch.ops.diffspec_b200 ops on the GPU: ``torch.library.opcheck``
(schema and mutation declarations, fake implementations, autograd
registration, AOT dispatch) with real CUDA inputs, and bit-equality with the
same call through the package's ctypes path."""

from __future__ import annotations

import importlib
from types import SimpleNamespace

import numpy as np
import pytest
import torch

import recipes as R

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops(dsb):
    importlib.import_module("vllm-ascend-hust-diffspec_b200.torch_ops")
    return torch.ops.diffspec_b200


def _opcheck(op, args):
    torch.library.opcheck(op, args, test_utils=("test_schema", "test_autograd_registration",
                                                "test_faketensor", "test_aot_dispatch_dynamic"))


def _paged(cuda, rows, length, hk, d, bs, seed):
    g = torch.Generator(device=cuda).manual_seed(seed)
    pages = (length + bs - 1) // bs
    kc = torch.randn((rows * pages, bs, hk, d), generator=g, device=cuda).bfloat16()
    table = torch.randperm(rows * pages, generator=g, device=cuda).view(rows, pages).int()
    return g, kc, table


def test_scores_op(dsb, ops, cuda):
    g, kc, table = _paged(cuda, 3, 700, 2, 128, 16, 1)
    q = torch.randn((3, 16, 128), generator=g, device=cuda).bfloat16()
    lse = torch.rand((3, 16), generator=g, device=cuda) + 4
    seq = torch.tensor([700, 333, 0], dtype=torch.int32, device=cuda)
    args = (q, kc, lse, table, seq, 32, 704, 128 ** -0.5)
    got = ops.paged_chunk_attention_scores(*args)
    ref = dsb.kernels.paged_chunk_attention_scores(q, kc, lse, table, seq, chunk_size=32,
                                                   max_seq_len=704, scale=128 ** -0.5)
    assert torch.equal(got, ref)
    _opcheck(ops.paged_chunk_attention_scores.default, args)


def test_gather_op(dsb, ops, cuda):
    inp = R.gather_inputs(0)
    bf = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda).bfloat16()  # noqa: E731
    args = (bf(inp["raw_key"]), bf(inp["raw_value"]), torch.from_numpy(inp["block_table"]).to(cuda),
            torch.from_numpy(inp["selected"]).to(cuda), bf(inp["cos_sin"]), inp["rot"], inp["neox"])
    k, v = ops.gather_raw_kv_with_local_rope(*args)
    rk, rv = dsb.kernels.gather_raw_kv_with_local_rope(*args[:5], rope_dim=inp["rot"],
                                                       is_neox_style=inp["neox"])
    assert torch.equal(k, rk) and torch.equal(v, rv)
    _opcheck(ops.gather_raw_kv_with_local_rope.default, args)


def _rebuild_state(cuda, window=0):
    g = torch.Generator(device=cuda).manual_seed(3)
    slots, max_len, hk, d, c, budget = 4, 900, 2, 128, 32, 512
    hb = (budget - 5) // c * c
    rk = torch.randn((slots, max_len, hk, d), generator=g, device=cuda).bfloat16()
    rv = torch.randn_like(rk)
    wk = torch.zeros((slots, hk, budget, d), device=cuda, dtype=torch.bfloat16)
    wv = torch.zeros_like(wk)
    inv = 1.0 / (1e6 ** (torch.arange(0, d, 2, device=cuda, dtype=torch.float64) / d))
    fr = torch.arange(budget, device=cuda, dtype=torch.float64)[:, None] * inv[None]
    cs = torch.cat((fr.cos(), fr.sin()), -1).to(torch.bfloat16).contiguous()
    row_slots = torch.tensor([2, 0, 3], dtype=torch.int32, device=cuda)
    committed = torch.tensor([890, 400, 77], dtype=torch.int32, device=cuda)
    sel_chunks = torch.zeros((slots, hb // c), dtype=torch.int32, device=cuda)
    sel_count = torch.full((slots,), -1, dtype=torch.int32, device=cuda)
    sel_chunks[2, :5] = torch.tensor([1, 5, 9, 20, 27], device=cuda)
    sel_count[2] = 5
    sel_count[0] = 0
    return dict(rk=rk, rv=rv, wk=wk, wv=wv, cs=cs, row_slots=row_slots, committed=committed,
                sel_chunks=sel_chunks, sel_count=sel_count, c=c, hb=hb, budget=budget, d=d)


def test_rebuild_ops(dsb, ops, cuda):
    s = _rebuild_state(cuda)
    width = 5 + s["budget"] // s["c"]
    for window in (0, 128):
        plan, hl, wl = (torch.zeros((3, width), dtype=torch.int64, device=cuda),
                        torch.zeros(3, dtype=torch.int32, device=cuda),
                        torch.zeros(4, dtype=torch.int32, device=cuda))
        wk, wv = s["wk"].clone(), s["wv"].clone()
        args = (s["rk"], s["rv"], wk, wv, s["row_slots"], s["committed"], s["sel_chunks"],
                s["sel_count"], s["cs"], plan, hl, wl, s["c"], s["hb"], s["d"], True, window)
        ops.rebuild_working_cache(*args)
        wk2, wv2 = s["wk"].clone(), s["wv"].clone()
        plan2, hl2 = dsb.compact_kv.rebuild_working_cache(
            s["rk"], s["rv"], wk2, wv2, s["row_slots"], s["committed"], s["sel_chunks"],
            s["sel_count"], s["cs"], chunk_size=s["c"], history_budget=s["hb"], rotary_dim=s["d"],
            is_neox_style=True, recent_window=window or None)
        assert torch.equal(plan, plan2) and torch.equal(hl, hl2)
        assert torch.equal(wk, wk2) and torch.equal(wv, wv2)
        _opcheck(ops.rebuild_working_cache.default, args)
        # the plan-driven op on the plan just computed
        wk3, wv3 = s["wk"].clone(), s["wv"].clone()
        pargs = (s["rk"], s["rv"], wk3, wv3, plan, s["cs"], s["c"], s["hb"], s["d"], True)
        ops.rebuild_compact_kv_from_plan(*pargs)
        assert torch.equal(wk3, wk2) and torch.equal(wv3, wv2)
        _opcheck(ops.rebuild_compact_kv_from_plan.default, pargs)
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0


def test_draft_attention_op(dsb, ops, cuda):
    g = torch.Generator(device=cuda).manual_seed(4)
    wk = torch.randn((4, 2, 256, 128), generator=g, device=cuda).bfloat16()
    wv = torch.randn_like(wk)
    q = torch.randn((5, 16, 128), generator=g, device=cuda).bfloat16()
    k = torch.randn((5, 2, 128), generator=g, device=cuda).bfloat16()
    v = torch.randn_like(k)
    slots = torch.tensor([3, 0, 2], dtype=torch.int32, device=cuda)
    pos = torch.tensor([100, 7, 250], dtype=torch.int32, device=cuda)
    out = torch.full_like(q, float("nan"))
    wk1, wv1 = wk.clone(), wv.clone()
    args = (q, k, v, wk1, wv1, slots, pos, 0.088, out, 3, 2)
    ops.draft_decode_attention(*args)
    wk2, wv2 = wk.clone(), wv.clone()
    ref = dsb.attention.draft_decode_attention(q, k, v, wk2, wv2, slots, pos, 0.088,
                                               torch.full_like(q, float("nan")), rows=3,
                                               position_offset=2)
    assert torch.equal(out, ref) and torch.equal(wk1, wk2) and torch.equal(wv1, wv2)
    assert not out[3:].any()
    _opcheck(ops.draft_decode_attention.default, args)
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0


def test_capture_op_drives_the_active_runtime(dsb, ops, cuda):
    t = importlib.import_module("vllm-ascend-hust-diffspec_b200.torch_ops")
    settings = dsb.runtime.DiffSpecSettings(8, 64, 1, 4, 3, 0.7, False)
    cache = dsb.runtime.DiffSpecDraftCache(
        settings, max_num_reqs=3, max_model_len=64, num_kv_heads=2, head_dim=64,
        target_num_layers=2, dtype=torch.bfloat16, device=cuda,
        cos_sin_cache=torch.zeros((64, 64), device=cuda))
    cache.raw_key.zero_()
    cache.raw_value.zero_()
    cache.set_active_requests(["a", "b"])
    cache.begin_cycle(["a", "b"])
    meta = SimpleNamespace(seq_lens_list=[30, 12])
    cache.prepare_compact_prefill(meta, 2, committed_seq_lens=[30, 12])
    t.set_active_runtime(cache)
    try:
        pos = torch.tensor([29, 11, 0, 0], device=cuda)
        key = torch.randn((4, 128), device=cuda).bfloat16()
        local = ops.capture_raw_kv(pos, key, key, 0)
        assert local.tolist() == [29, 11, 0, 0]  # history lengths (no retrieval yet), padding 0
        assert torch.equal(cache.raw_key[0, 29].reshape(-1), key[0])
        assert torch.equal(cache.raw_key[1, 11].reshape(-1), key[1])
        assert not cache.raw_key[:, 0].any()  # padding rows wrote nothing
        _opcheck(ops.capture_raw_kv.default, (pos, key, key, 0))
    finally:
        t.set_active_runtime(None)
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0
