"""Pin the oracle's chains against the reference run end to end
(tests/golden/make_golden.py: make_config1, make_capture).

* BASELINE config 1 (one request, 4096 tokens, chunk 32, budget 512, 1 / 8
  heads of 128, fp32, 4 planted chunks, last 3 draft tokens rejected):
  chunk_attention_scores -> select_context_chunks -> _rebuild_working_cache
  -> forward_attention (diffspec/runtime.py:281-345, 348-414, 1683-1711,
  2040-2077).
* The draft step's KV sink: populate_prefill, a retrieval, then
  prepare_compact_prefill and capture_raw_kv + forward_attention per draft
  step with graph-padding rows in reordered slots (runtime.py:1336-1371,
  1602-1618, 1797-1877).
* Request slots: set_active_requests over a sequence of batches (reorder,
  cancellation, a returning id, duplicates, exhaustion; runtime.py:755-778)."""

from __future__ import annotations

import numpy as np

import recipes as R
from conftest import golden
from oracle import diffspec_oracle as O


def test_config1_chain_matches_reference():
    d, c, inp = golden("config1"), R.CONFIG1, R.config1_inputs()
    assert int(d["crc"]) == R.crc(inp["keys"], inp["values"], inp["query"])
    L, hb = inp["retrieval_len"], int(d["history_budget"])
    assert hb == O.history_budget(c["budget"], c["depth"], c["chunk"])
    scale = c["d"] ** -0.5
    scores = O.chunk_attention_scores(inp["query"], inp["keys"][:L], c["chunk"], None, scale)
    np.testing.assert_allclose(scores, d["scores"], rtol=1e-4, atol=1e-9)
    ci, ti, _ = O.select_context_chunks(d["scores"], L, c["chunk"], hb)
    np.testing.assert_array_equal(ci, d["chunk_indices"])
    np.testing.assert_array_equal(ti, d["token_indices"])
    assert set(c["planted"]) <= set(ci.tolist())
    assert O.selection_margin(d["scores"], L, c["chunk"], hb) > 1e-3  # no near-tie at the cut
    row = O.history_plan(0, ci.tolist(), inp["committed"] - 1, c["chunk"], hb)
    np.testing.assert_array_equal(row, d["plan"])
    assert row[1] == int(d["local_positions"][0])
    plan = np.zeros((1, 5 + c["budget"] // c["chunk"]), np.int64)
    plan[0, : len(row)] = row
    wk = np.zeros((1, c["hk"], c["budget"], c["d"]), np.float32)
    wv = np.zeros_like(wk)
    O.rebuild_compact_kv_from_plan(inp["keys"][None], inp["values"][None], wk, wv, plan,
                                   inp["cos_sin"], c["chunk"], hb, c["d"], True, "f32")
    h = row[1]
    np.testing.assert_array_equal(wk[0, :, :h], d["working_key"])  # fp32 RoPE, bit for bit
    st = inp["steps"]
    for j in range(c["depth"]):
        out = O.draft_decode_attention(st["query"][j], st["key"][j], st["value"][j], wk, wv, [0],
                                       [h + j], scale, dtype=None)
        np.testing.assert_allclose(out, d[f"step{j}_out"], rtol=1e-5, atol=1e-6)
    assert int(d["working_lens"][0]) == h + c["depth"]


def test_capture_cycle_matches_reference():
    d, c, inp = golden("capture"), R.CAPTURE, R.capture_inputs()
    assert int(d["crc"]) == R.crc(inp["prefill_key"], inp["prefill_value"], inp["mid_scores"])
    slots = d["active_slots"].tolist()
    assert slots == [3, 1, 2]
    hk, dim, S = c["hk"], c["d"], c["slots"]
    raw_k = np.zeros((S, c["max_len"], hk, dim), np.float32)
    raw_v = np.zeros_like(raw_k)
    rows = O.request_rows(inp["query_ends"], len(inp["prefill_positions"]))
    O.write_raw(raw_k, raw_v, [slots[r] for r in rows], inp["prefill_positions"],
                inp["prefill_key"], inp["prefill_value"])
    hb = O.history_budget(c["budget"], c["depth"], c["chunk"])
    prompts = list(c["prompts"])
    mid = O.select_context_chunks(inp["mid_scores"], prompts[1], c["chunk"], hb)[0]
    np.testing.assert_array_equal(mid, d["mid_chunks"])
    sel = {slots[1]: mid.tolist()}
    width = 5 + c["budget"] // c["chunk"]
    plan = np.zeros((len(slots), width), np.int64)
    for r, slot in enumerate(slots):
        row = O.history_plan(slot, sel.get(slot), prompts[r], c["chunk"], hb)
        plan[r, : len(row)] = row
    wk = np.zeros((S, hk, c["budget"], dim), np.float32)
    wv = np.zeros_like(wk)
    O.rebuild_compact_kv_from_plan(raw_k, raw_v, wk, wv, plan, inp["cos_sin"], c["chunk"], hb,
                                   dim, True, "f32")
    for j, st in enumerate(inp["steps"]):
        local = O.capture_raw_kv(raw_k, raw_v, slots, st["positions"], st["key"], st["value"],
                                 plan[:, 1], j)
        np.testing.assert_array_equal(local, d[f"step{j}_local_positions"])
        out = O.draft_decode_attention(st["query"], st["key"], st["value"], wk, wv, slots,
                                       local[: len(slots)], dim ** -0.5, dtype=None)
        np.testing.assert_allclose(out, d[f"step{j}_out"], rtol=1e-5, atol=1e-6)
    np.testing.assert_array_equal(raw_k, d["raw_key"])
    np.testing.assert_array_equal(raw_v, d["raw_value"])
    for r, slot in enumerate(slots):
        h = int(plan[r, 1]) + c["depth"]
        np.testing.assert_array_equal(wk[slot, :, :h], d["working_key"][slot, :, :h])
        np.testing.assert_array_equal(wv[slot, :, :h], d["working_value"][slot, :, :h])
        assert int(d["working_lens"][slot]) == h


def slot_step_state(table: O.SlotTable, d: dict, i: int) -> None:
    """Compare the oracle's slot table after step i with the reference's."""
    assert table.active == d[f"active{i}"].tolist()
    assert table.working_lens == d[f"working_lens{i}"].tolist()
    assert sorted(table.selected) == np.flatnonzero(d[f"selected{i}"]).tolist()


def test_slot_table_matches_reference():
    d = golden("slots")
    assert int(d["n"]) == len(R.SLOT_STEPS)
    table = O.SlotTable(R.SLOT_COUNT)
    for i, batch in enumerate(R.SLOT_STEPS):
        for slot in table.slots.values():
            table.working_lens[slot] = 100 + 10 * i + slot
            table.selected.add(slot)
        raised = 0
        try:
            table.set_active_requests(list(batch))
        except RuntimeError:
            raised = 1
        assert raised == int(d[f"raised{i}"])
        slot_step_state(table, d, i)
