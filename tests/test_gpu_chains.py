"""Whole chains through DiffSpecDraftCache on the GPU against the reference
run end to end (tests/golden/config1.npz, capture.npz; make_golden.py):

* BASELINE config 1 (reference mode and, against the oracle, the 128-token
  window mode): scores -> selection -> plan + rebuild -> 4 draft steps;
* the KV sink: populate_prefill, a retrieval, prepare_compact_prefill, then
  capture_raw_kv + forward_attention per step with graph-padding rows in
  reordered slots;
* the raw-KV write (dsb_write_raw_kv, DiffSpecDraftCache.write_raw) against
  _write_raw (diffspec/runtime.py:1602-1618).

The reference runs these chains in fp32 (its CPU attention loop needs fp32
caches) on values exact in bf16; here the caches are bf16, so chunk ids,
plans, local positions and raw-cache rows must be bit-exact and the rebuilt
K must equal the reference's fp32 RoPE rounded once to bf16.  Attention
outputs must meet the bf16 tolerance (max abs error <= 2e-2, mean <= 2e-3
relative) against the oracle evaluated over the same bf16 working cache
(the oracle itself matches the reference's fp32 run to 1e-5,
test_oracle_chains.py); against the reference's fp32-cache outputs directly
the mean bound is 4e-3, since the bf16 rounding of every rotated key adds
about as much error as the bf16 rounding of the output."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import recipes as R
from conftest import close_bf16, golden
from oracle import diffspec_oracle as O

pytestmark = pytest.mark.gpu

FP32_CACHE_MEAN_REL = 4e-3  # GPU (bf16 working cache) against the reference's fp32 cache


def _bf(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev).bfloat16()


def _config1_cache(dsb, cuda, window=None):
    c, inp = R.CONFIG1, R.config1_inputs()
    settings = dsb.runtime.DiffSpecSettings(c["chunk"], c["budget"], 1, 4, c["depth"], 0.7, False)
    cache = dsb.runtime.DiffSpecDraftCache(
        settings, max_num_reqs=1, max_model_len=c["tokens"], num_kv_heads=c["hk"], head_dim=c["d"],
        target_num_layers=2, dtype=torch.bfloat16, device=cuda,
        cos_sin_cache=torch.from_numpy(inp["cos_sin"]).to(cuda), rotary_dim=c["d"],
        is_neox_style=True, recent_window=window)
    cache.raw_key[0] = _bf(inp["keys"], cuda)
    cache.raw_value[0] = _bf(inp["values"], cuda)
    return cache, c, inp


def test_config1_chain_vs_reference(dsb, cuda):
    d = golden("config1")
    cache, c, inp = _config1_cache(dsb, cuda)
    L, scale = inp["retrieval_len"], c["d"] ** -0.5
    assert cache.history_budget == int(d["history_budget"])
    scores = dsb.runtime.chunk_attention_scores(_bf(inp["query"], cuda), _bf(inp["keys"][:L], cuda),
                                                c["chunk"], None, scale)
    np.testing.assert_allclose(scores.cpu().numpy(), d["scores"], rtol=1e-3, atol=1e-9)
    cache.begin_cycle(["r"])
    sel = cache.set_chunk_scores(0, scores, L)
    np.testing.assert_array_equal(sel.chunk_indices.cpu().numpy(), d["chunk_indices"])
    np.testing.assert_array_equal(sel.token_indices.cpu().numpy(), d["token_indices"])
    hl = cache.rebuild([inp["committed"]])
    h = int(d["local_positions"][0])
    assert int(hl[0]) == h
    plan = d["plan"]
    np.testing.assert_array_equal(cache._plan[0, : plan.size].cpu().numpy(), plan)
    wk = cache.working_key[0, :, :h].float().cpu().numpy()
    np.testing.assert_array_equal(wk, O.round_to(d["working_key"], "bf16"))
    idx = O.decode_history_plan(plan, c["chunk"])
    np.testing.assert_array_equal(cache.working_value[0, :, :h].float().cpu().numpy(),
                                  inp["values"][idx].transpose(1, 0, 2))
    st = inp["steps"]
    ok = np.zeros((1, c["hk"], c["budget"], c["d"]), np.float32)  # the oracle over the bf16 cache
    ov = np.zeros_like(ok)
    ok[0, :, :h] = wk
    ov[0, :, :h] = inp["values"][idx].transpose(1, 0, 2)
    out = torch.empty((1, c["hq"], c["d"]), dtype=torch.bfloat16, device=cuda)
    for j in range(c["depth"]):
        cache.forward_attention(_bf(st["query"][j], cuda), _bf(st["key"][j], cuda),
                                _bf(st["value"][j], cuda), scale, out)
        got = out.float().cpu().numpy()
        ref = O.draft_decode_attention(st["query"][j], st["key"][j], st["value"][j], ok, ov, [0],
                                       [h + j], scale, dtype=None)
        close_bf16(got, ref)
        close_bf16(got, d[f"step{j}_out"], mean_rel=FP32_CACHE_MEAN_REL)
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0


def test_config1_chain_window_mode_vs_oracle(dsb, cuda):
    """Config 1's 128-token recent window: the same chain in window mode
    against the oracle's restatement of the mode."""
    cache, c, inp = _config1_cache(dsb, cuda, window=c1_window())
    L, scale, hb, w = inp["retrieval_len"], c["d"] ** -0.5, cache.history_budget, c1_window()
    scores = dsb.runtime.chunk_attention_scores(_bf(inp["query"], cuda), _bf(inp["keys"][:L], cuda),
                                                c["chunk"], None, scale)
    ref_scores = O.chunk_attention_scores(inp["query"], inp["keys"][:L], c["chunk"], None, scale)
    assert O.selection_margin(ref_scores, L, c["chunk"], hb, recent_window=w) > 1e-4
    cache.begin_cycle(["r"])
    sel = cache.set_chunk_scores(0, scores, L)
    ci = O.select_context_chunks(ref_scores, L, c["chunk"], hb, recent_window=w)[0]
    np.testing.assert_array_equal(sel.chunk_indices.cpu().numpy(), ci)
    assert set(c["planted"]) <= set(ci.tolist())
    hl = cache.rebuild([inp["committed"]])
    row = O.history_plan(0, ci.tolist(), inp["committed"] - 1, c["chunk"], hb, recent_window=w)
    np.testing.assert_array_equal(cache._plan[0, : len(row)].cpu().numpy(), row)
    h = row[1]
    assert int(hl[0]) == h == hb and row[3] == hb - w  # the prefix fills what the window leaves
    plan = np.zeros((1, 5 + c["budget"] // c["chunk"]), np.int64)
    plan[0, : len(row)] = row
    wk = np.zeros((1, 1, c["budget"], c["d"]), np.float32)
    wv = np.zeros_like(wk)
    O.rebuild_compact_kv_from_plan(inp["keys"][None], inp["values"][None], wk, wv, plan,
                                   inp["cos_sin"], c["chunk"], hb, c["d"], True, "bf16")
    np.testing.assert_array_equal(cache.working_key[:1, :, :h].float().cpu().numpy(), wk[:, :, :h])
    st = inp["steps"]
    out = torch.empty((1, c["hq"], c["d"]), dtype=torch.bfloat16, device=cuda)
    for j in range(c["depth"]):
        cache.forward_attention(_bf(st["query"][j], cuda), _bf(st["key"][j], cuda),
                                _bf(st["value"][j], cuda), scale, out)
        ref = O.draft_decode_attention(st["query"][j], st["key"][j], st["value"][j], wk, wv, [0],
                                       [h + j], scale, dtype=None)
        close_bf16(out.float().cpu().numpy(), ref)
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0


def c1_window() -> int:
    return R.CONFIG1["window"]


def test_capture_cycle_vs_reference(dsb, cuda):
    d, c, inp = golden("capture"), R.CAPTURE, R.capture_inputs()
    from types import SimpleNamespace

    settings = dsb.runtime.DiffSpecSettings(c["chunk"], c["budget"], 1, 4, c["depth"], 0.7, False)
    cache = dsb.runtime.DiffSpecDraftCache(
        settings, max_num_reqs=c["slots"], max_model_len=c["max_len"], num_kv_heads=c["hk"],
        head_dim=c["d"], target_num_layers=2, dtype=torch.bfloat16, device=cuda,
        cos_sin_cache=_bf(inp["cos_sin"], cuda), rotary_dim=c["d"], is_neox_style=True)
    cache.raw_key.zero_()
    cache.raw_value.zero_()
    ids = ["c", "a", "b"]
    cache.set_active_requests(["x", "a", "b", "c"])
    cache.set_active_requests(ids)
    slots = cache.active_slots()
    assert slots == d["active_slots"].tolist()
    cache.populate_prefill(torch.from_numpy(inp["prefill_positions"]).to(cuda),
                           _bf(inp["prefill_key"], cuda), _bf(inp["prefill_value"], cuda),
                           SimpleNamespace(actual_seq_lengths_q=inp["query_ends"].tolist()))
    prompts = list(c["prompts"])
    sel = cache.set_chunk_scores(slots[1], torch.from_numpy(inp["mid_scores"]).to(cuda),
                                 prompts[1])
    np.testing.assert_array_equal(sel.chunk_indices.cpu().numpy(), d["mid_chunks"])
    cache.begin_cycle(ids)
    committed = [n + 1 for n in prompts]
    meta = SimpleNamespace(seq_lens_list=committed, actual_seq_lengths_q=[1, 2, 3])
    cache.prepare_compact_prefill(meta, len(ids), committed_seq_lens=committed)
    held = []
    # the oracle over the GPU's bf16 working cache, rebuilt from the reference's fp32 one
    ok = np.zeros_like(d["working_key"])
    ov = np.zeros_like(ok)
    for slot in slots:
        h0 = int(d["working_lens"][slot]) - c["depth"]  # the plan's history length
        ok[slot, :, :h0] = O.round_to(d["working_key"][slot, :, :h0], "bf16")
        ov[slot, :, :h0] = d["working_value"][slot, :, :h0]
    for j, st in enumerate(inp["steps"]):
        pos = torch.from_numpy(st["positions"]).to(cuda)
        local = cache.capture_raw_kv(0, pos, _bf(st["key"], cuda), _bf(st["value"], cuda))
        assert local.shape == pos.shape and local.dtype == pos.dtype
        np.testing.assert_array_equal(local.cpu().numpy(), d[f"step{j}_local_positions"])
        same = cache.graph_safe_rope_positions(pos, local)
        assert same.data_ptr() == local.data_ptr()  # the sink's buffer is already cache-owned
        held.append(local.data_ptr())
        out = torch.full((len(st["positions"]), c["hq"], c["d"]), float("nan"), device=cuda,
                         dtype=torch.bfloat16)
        cache.forward_attention(_bf(st["query"], cuda), _bf(st["key"], cuda), _bf(st["value"], cuda),
                                c["d"] ** -0.5, out)
        got = out.float().cpu().numpy()
        ref = O.draft_decode_attention(st["query"], st["key"], st["value"], ok, ov,
                                       slots, local.cpu().numpy()[: len(ids)],
                                       c["d"] ** -0.5, dtype=None)
        close_bf16(got[: len(ids)], ref[: len(ids)])
        close_bf16(got[: len(ids)], d[f"step{j}_out"][: len(ids)], mean_rel=FP32_CACHE_MEAN_REL)
        assert not got[len(ids):].any()  # padding rows are zero
    assert len(set(held)) == 1  # one stable position buffer for every step
    # the working lengths advance with the steps, as forward_attention's do
    np.testing.assert_array_equal(cache.working_lens.cpu().numpy(), d["working_lens"])
    cache.end_cycle()
    np.testing.assert_array_equal(cache.raw_key.float().cpu().numpy(), d["raw_key"])
    np.testing.assert_array_equal(cache.raw_value.float().cpu().numpy(), d["raw_value"])
    for slot in slots:
        h = int(d["working_lens"][slot])
        np.testing.assert_array_equal(cache.working_key[slot, :, :h].float().cpu().numpy(),
                                      O.round_to(d["working_key"][slot, :, :h], "bf16"))
        np.testing.assert_array_equal(cache.working_value[slot, :, :h].float().cpu().numpy(),
                                      d["working_value"][slot, :, :h])
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0


def test_capture_positions_buffer_and_prefill_path(dsb, cuda):
    """graph_safe_rope_positions keeps one buffer per dtype and clears what a
    longer earlier call left; capture_raw_kv outside a cycle writes like
    populate_prefill and returns nothing."""
    from types import SimpleNamespace

    settings = dsb.runtime.DiffSpecSettings(8, 64, 1, 4, 3, 0.7, False)
    table = torch.zeros((64, 64), device=cuda)
    cache = dsb.runtime.DiffSpecDraftCache(
        settings, max_num_reqs=2, max_model_len=32, num_kv_heads=1, head_dim=64,
        target_num_layers=2, dtype=torch.bfloat16, device=cuda, cos_sin_cache=table)
    a = cache.graph_safe_rope_positions(torch.arange(10, 20, device=cuda), None)
    assert a.tolist() == list(range(10, 20))
    b = cache.graph_safe_rope_positions(torch.arange(3, device=cuda), None)
    assert b.data_ptr() == a.data_ptr() and b.tolist() == [0, 1, 2]
    assert cache._position_buffers[torch.int64][:10].tolist() == [0, 1, 2] + [0] * 7
    cache.raw_key.zero_()
    cache.raw_value.zero_()
    cache.set_active_requests(["p", "q"])
    k = torch.randn((5, 1, 64), device=cuda).bfloat16()
    pos = torch.tensor([0, 1, 2, 0, 1], device=cuda)
    meta = SimpleNamespace(actual_seq_lengths_q=[3, 5])
    assert cache.capture_raw_kv(0, pos, k, k, meta) is None
    assert torch.equal(cache.raw_key[0, :3], k[:3]) and torch.equal(cache.raw_key[1, :2], k[3:])
    with pytest.raises(ValueError):
        cache.capture_raw_kv(1, pos, k, k, meta)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_write_raw_vs_reference_write(dsb, cuda, dtype):
    """dsb_write_raw_kv / DiffSpecDraftCache.write_raw against _write_raw:
    rows land at [slot, position], padding rows (slot -1) write nothing,
    every other row is untouched, and bad slots / positions are flagged and
    skipped."""
    g = R.rng(31)
    slots_n, max_len, hk, d, n = 4, 50, 2, 64, 40
    settings = dsb.runtime.DiffSpecSettings(8, 64, 1, 4, 3, 0.7, False)
    cache = dsb.runtime.DiffSpecDraftCache(
        settings, max_num_reqs=slots_n, max_model_len=max_len, num_kv_heads=hk, head_dim=d,
        target_num_layers=2, dtype=dtype, device=cuda, cos_sin_cache=torch.zeros((64, d), device=cuda))
    base_k = O.round_to(g.standard_normal((slots_n, max_len, hk, d), dtype=np.float32), "bf16")
    base_v = O.round_to(g.standard_normal((slots_n, max_len, hk, d), dtype=np.float32), "bf16")
    cache.raw_key.copy_(torch.from_numpy(base_k).to(cuda, dtype))
    cache.raw_value.copy_(torch.from_numpy(base_v).to(cuda, dtype))
    flat = g.permutation(slots_n * max_len)[:n]
    slots = (flat // max_len).astype(np.int32)
    positions = (flat % max_len).astype(np.int64)
    slots[::7] = -1  # padding rows
    key = O.round_to(g.standard_normal((n, hk, d), dtype=np.float32), "bf16")
    value = O.round_to(g.standard_normal((n, hk, d), dtype=np.float32), "bf16")
    cache.write_raw(torch.from_numpy(slots).to(cuda), torch.from_numpy(positions).to(cuda),
                    torch.from_numpy(key).to(cuda, dtype), torch.from_numpy(value).to(cuda, dtype))
    ref_k, ref_v = base_k.copy(), base_v.copy()
    O.write_raw(ref_k, ref_v, slots, positions, key, value)
    np.testing.assert_array_equal(cache.raw_key.float().cpu().numpy(), ref_k)
    np.testing.assert_array_equal(cache.raw_value.float().cpu().numpy(), ref_v)
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0
    # a slot and a position out of range: flagged, the other rows still written
    bad_slots = torch.tensor([0, slots_n, 1], dtype=torch.int32, device=cuda)
    bad_pos = torch.tensor([3, 4, max_len], dtype=torch.int64, device=cuda)
    kk = torch.ones((3, hk, d), device=cuda, dtype=dtype)
    cache.write_raw(bad_slots, bad_pos, kk, kk)
    flag = dsb._lib.read_and_clear_error_flag(cuda)
    assert flag & 1 and flag & 2  # DSB_FLAG_SLOT, DSB_FLAG_POSITION
    assert bool((cache.raw_key[0, 3] == 1).all())
    np.testing.assert_array_equal(cache.raw_key[1].float().cpu().numpy(), ref_k[1])
