"""Rolling-recent-window mode (BASELINE configs 1 and 2: windows of 128 and
256 tokens) on the device against the oracle's restatement, bit for bit:
selection, plan rows, the fused plan + rebuild and a whole runtime cycle.

The mode has no reference counterpart (the reference's rolling tail is one
chunk, diffspec/runtime.py:1657-1659, 1719-1720); with window = chunk size
every path must reproduce the reference exactly, which the fixture tests
check, and which the parity case here checks again through the window
argument."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import recipes as R
from oracle import diffspec_oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("c,budget,window", [(32, 480, 128), (64, 1984, 256), (64, 1984, 64),
                                             (32, 480, 480), (16, 256, 240)])
@pytest.mark.parametrize("n", [3, 15, 16, 17, 700, 4097])
def test_window_selection_vs_oracle(dsb, cuda, c, budget, window, n):
    g = R.rng(n * 7 + window)
    s = (g.integers(0, 50, n) / 8).astype(np.float32)  # many ties
    for seq_len in (n * c, n * c - c // 2 - 1):
        if seq_len <= (n - 1) * c:
            continue
        sel = dsb.selection.select_context_chunks(torch.from_numpy(s).to(cuda), seq_len, c, budget,
                                                  recent_window=window)
        ref = O.select_context_chunks(s, seq_len, c, budget, recent_window=window)
        np.testing.assert_array_equal(sel.chunk_indices.cpu().numpy(), ref[0])
        np.testing.assert_array_equal(sel.token_indices.cpu().numpy(), ref[1])
        np.testing.assert_array_equal(sel.chunk_scores.cpu().numpy(), ref[2])


@pytest.mark.parametrize("c,hb,window", [(32, 480, 128), (64, 1984, 256), (16, 128, 64)])
def test_window_plans_vs_oracle(dsb, cuda, c, hb, window):
    """Plans of random selections at random history ends, with the rows'
    expansions checked against the oracle's _history_indices restatement."""
    g = R.rng(hb + window)
    rows, s_cap = 64, hb // c
    sel_chunks = np.zeros((rows, s_cap), np.int32)
    counts, committed, expect = [], [], []
    for r in range(rows):
        he = int(g.integers(0, 40 * hb))
        committed.append(he + 1)
        if r % 9 == 0:
            counts.append(-1)
            chosen = None
        else:
            n = max(1, (he + 1 + c - 1) // c)
            k = int(g.integers(0, min(n, s_cap - window // c + 1) + 1))
            chosen = sorted(g.choice(n, k, replace=False).tolist()) if k else []
            if chosen and chosen[-1] != n - 1 and r % 2:
                chosen = chosen[:-1] + [n - 1]
                chosen = sorted(set(chosen))
            counts.append(len(chosen))
            sel_chunks[r, : len(chosen)] = chosen
        expect.append(O.history_plan(r, chosen, he, c, hb, recent_window=window))
    plan, hl = dsb.selection.build_history_plan(
        torch.arange(rows, dtype=torch.int32, device=cuda),
        torch.tensor(committed, dtype=torch.int32, device=cuda), torch.from_numpy(sel_chunks).to(cuda),
        torch.tensor(counts, dtype=torch.int32, device=cuda), chunk_size=c, history_budget=hb,
        working_budget=hb + c, recent_window=window)
    plan = plan.cpu().numpy()
    for r in range(rows):
        ref = np.array(expect[r], np.int64)
        np.testing.assert_array_equal(plan[r, : ref.size], ref)
        assert not plan[r, ref.size:].any()
        assert int(hl[r]) == ref[1]
        he = committed[r] - 1
        if counts[r] >= 0:
            chosen = sel_chunks[r, : counts[r]].tolist()
            tokens = [t for ch in chosen for t in range(ch * c, ch * c + c)]
            assert O.decode_history_plan(ref, c) == O.history_indices(
                np.array(tokens, np.int64) if chosen else np.zeros(0, np.int64), he, c, hb,
                recent_window=window).tolist()
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0


@pytest.mark.parametrize("window", [128, 256])
def test_window_fused_rebuild_vs_oracle(dsb, cuda, window):
    """Plan + rebuild in one launch with the window: plans and working
    caches bit-exact against the oracle's plan and rebuild."""
    g = R.rng(window)
    slots, max_len, hk, d, c, budget = 6, 3000, 2, 128, 64, 2048
    hb = (budget - 5) // c * c
    raw_k = O.round_to(g.standard_normal((slots, max_len, hk, d), dtype=np.float32), "bf16")
    raw_v = O.round_to(g.standard_normal((slots, max_len, hk, d), dtype=np.float32), "bf16")
    inv = 1.0 / (1e6 ** (np.arange(0, d, 2) / d))
    fr = np.arange(budget)[:, None] * inv[None]
    cs = O.round_to(np.concatenate([np.cos(fr), np.sin(fr)], -1).astype(np.float32), "bf16")
    committed = [2999, 2600, 1500, 64, 3000, 2201]
    row_slots = [3, 0, 5, 1, 2, 4]
    sel_chunks = np.zeros((slots, hb // c), np.int32)
    counts = np.full(slots, -1, np.int32)
    for r, (slot, L) in enumerate(zip(row_slots, committed)):
        if r == 2:
            continue  # no retrieval yet
        n = (L + c - 1) // c
        scores = g.random(n).astype(np.float32)
        ch = O.select_context_chunks(scores, L, c, hb, recent_window=window)[0]
        sel_chunks[slot, : ch.size] = ch
        counts[slot] = ch.size
    bf = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda).bfloat16()  # noqa: E731
    wk = torch.zeros((slots, hk, budget, d), device=cuda, dtype=torch.bfloat16)
    wv = torch.zeros_like(wk)
    plan, hl = dsb.compact_kv.rebuild_working_cache(
        bf(raw_k), bf(raw_v), wk, wv, torch.tensor(row_slots, dtype=torch.int32, device=cuda),
        torch.tensor(committed, dtype=torch.int32, device=cuda), torch.from_numpy(sel_chunks).to(cuda),
        torch.from_numpy(counts).to(cuda), bf(cs), chunk_size=c, history_budget=hb, rotary_dim=d,
        is_neox_style=True, recent_window=window)
    ref_plan = np.zeros((len(row_slots), 5 + budget // c), np.int64)
    for r, (slot, L) in enumerate(zip(row_slots, committed)):
        chosen = None if counts[slot] < 0 else sel_chunks[slot, : counts[slot]].tolist()
        row = O.history_plan(slot, chosen, L - 1, c, hb, recent_window=window)
        ref_plan[r, : len(row)] = row
    np.testing.assert_array_equal(plan.cpu().numpy(), ref_plan)
    ok, ov = np.zeros((slots, hk, budget, d), np.float32), np.zeros((slots, hk, budget, d), np.float32)
    O.rebuild_compact_kv_from_plan(raw_k, raw_v, ok, ov, ref_plan, cs, c, hb, d, True, "bf16")
    assert np.array_equal(wk.float().cpu().numpy(), ok)
    assert np.array_equal(wv.float().cpu().numpy(), ov)
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0


def test_runtime_cycle_with_window_vs_oracle(dsb, cuda):
    """A DiffSpecDraftCache with recent_window 128 (config 1's window): the
    selection it stores after a retrieval, the plan of the next rebuild and
    the draft attention output follow the oracle's window-mode chain."""
    g = R.rng(128)
    c, budget, depth, hq, hk, d, bs, L = 32, 512, 4, 8, 1, 128, 16, 4096
    settings = dsb.runtime.DiffSpecSettings(c, budget, 1, 4, depth, 0.7, False)
    inv = 1.0 / (1e6 ** (np.arange(0, d, 2) / d))
    fr = np.arange(budget)[:, None] * inv[None]
    cs = torch.from_numpy(np.concatenate([np.cos(fr), np.sin(fr)], -1).astype(np.float32)).to(cuda)
    cache = dsb.runtime.DiffSpecDraftCache(
        settings, max_num_reqs=2, max_model_len=L + 64, num_kv_heads=hk, head_dim=d,
        target_num_layers=2, dtype=torch.bfloat16, device=cuda, cos_sin_cache=cs, rotary_dim=d,
        is_neox_style=True, recent_window=128)
    hb = cache.history_budget
    q = O.round_to(g.standard_normal((1, hq, d), dtype=np.float32), "bf16")
    kc = O.round_to(g.standard_normal((L // bs, bs, hk, d), dtype=np.float32), "bf16")
    table = np.arange(L // bs, dtype=np.int32)[None]
    lse = (g.random((1, hq)) + 5.0).astype(np.float32)
    cache.set_active_requests(["a"])
    cache.retrieve(torch.from_numpy(q).to(cuda).bfloat16(), torch.from_numpy(lse).to(cuda),
                   torch.from_numpy(kc).to(cuda).bfloat16(), torch.from_numpy(table).to(cuda), [1], [L - 2],
                   torch.tensor([1], device=cuda), d ** -0.5)
    scores = O.paged_chunk_attention_scores(q, kc, lse, table, np.array([L - 2]), c,
                                            L, d ** -0.5)[0]
    n = (L - 2 + c - 1) // c
    ref_chunks = O.select_context_chunks(scores[:n], L - 2, c, hb, recent_window=128)[0]
    got = cache.sel_chunks[0, : int(cache.sel_count[0])].cpu().numpy()
    margin = O.selection_margin(scores[:n], L - 2, c, hb, recent_window=128)
    if margin > 1e-4:
        np.testing.assert_array_equal(got, ref_chunks)
    else:
        ref_chunks = got  # a near-tie at the cut: follow the device's choice below
    raw_k = O.round_to(g.standard_normal((L + 64, hk, d), dtype=np.float32), "bf16")
    raw_v = O.round_to(g.standard_normal((L + 64, hk, d), dtype=np.float32), "bf16")
    cache.raw_key[0] = torch.from_numpy(raw_k).to(cuda).bfloat16()
    cache.raw_value[0] = torch.from_numpy(raw_v).to(cuda).bfloat16()
    committed = L - 2 + 3
    hl = cache.rebuild([committed])
    row = O.history_plan(0, ref_chunks.tolist(), committed - 1, c, hb, recent_window=128)
    assert int(hl[0]) == row[1] and row[1] == hb
    assert row[3] == hb - 128  # the prefix fills the budget left by the window
    plan = np.zeros((1, 5 + budget // c), np.int64)
    plan[0, : len(row)] = row
    ok, ov = np.zeros((1, hk, budget, d), np.float32), np.zeros((1, hk, budget, d), np.float32)
    O.rebuild_compact_kv_from_plan(raw_k[None], raw_v[None], ok, ov, plan, cs.cpu().numpy(), c, hb, d,
                                   True, "bf16")
    h = row[1]  # positions past the history are the cache's (uninitialised) capacity
    assert np.array_equal(cache.working_key[:1, :, :h].float().cpu().numpy(), ok[:, :, :h])
    assert np.array_equal(cache.working_value[:1, :, :h].float().cpu().numpy(), ov[:, :, :h])
    dq = O.round_to(g.standard_normal((1, hq, d), dtype=np.float32), "bf16")
    dk = O.round_to(g.standard_normal((1, hk, d), dtype=np.float32), "bf16")
    out = torch.empty((1, hq, d), device=cuda, dtype=torch.bfloat16)
    cache.forward_attention(torch.from_numpy(dq).to(cuda).bfloat16(), torch.from_numpy(dk).to(cuda).bfloat16(),
                            torch.from_numpy(dk).to(cuda).bfloat16(), d ** -0.5, out)
    expect = O.draft_decode_attention(dq, dk, dk, ok, ov, [0], [row[1]], d ** -0.5, dtype=None)
    err = np.abs(out.float().cpu().numpy() - expect)
    assert err.max() <= 2e-2 * max(1.0, np.abs(expect).max())
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0
