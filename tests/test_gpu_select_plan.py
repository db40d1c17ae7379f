"""Device top-k selection (A4) and compact history plans (A5): bit-exact."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import recipes as R
from conftest import golden
from oracle import diffspec_oracle as O

pytestmark = pytest.mark.gpu


def test_select_matches_reference_exactly(dsb, cuda):
    d = golden("select")
    for i, (seq_len, c, budget) in enumerate(R.select_cases()):
        n = (seq_len + c - 1) // c
        scores = torch.from_numpy(R.select_scores(i, n)).to(cuda)
        sel = dsb.selection.select_context_chunks(scores, seq_len, c, budget)
        np.testing.assert_array_equal(sel.chunk_indices.cpu().numpy(), d[f"case{i}_chunk_indices"])
        np.testing.assert_array_equal(sel.token_indices.cpu().numpy(), d[f"case{i}_token_indices"])
        np.testing.assert_array_equal(sel.chunk_scores.cpu().numpy(),
                                      R.select_scores(i, n)[d[f"case{i}_chunk_indices"]])


@pytest.mark.parametrize("pattern", ["all_equal", "blocks", "quantized", "zeros_and_inf"])
def test_ties_go_to_the_lower_chunk_index(dsb, cuda, pattern):
    g = R.rng(77)
    n, c, budget = 700, 32, 32 * 31
    if pattern == "all_equal":
        s = np.full(n, 0.25, np.float32)
    elif pattern == "blocks":
        s = np.repeat(g.random(35).astype(np.float32), 20)
    elif pattern == "quantized":
        s = (g.integers(0, 4, n) / 4).astype(np.float32)
    else:
        s = np.zeros(n, np.float32)
        s[g.choice(n, 10, replace=False)] = np.inf
    seq_len = n * c - 5
    sel = dsb.selection.select_context_chunks(torch.from_numpy(s).to(cuda), seq_len, c, budget)
    ref = O.select_context_chunks(s, seq_len, c, budget)
    np.testing.assert_array_equal(sel.chunk_indices.cpu().numpy(), ref[0])
    np.testing.assert_array_equal(sel.token_indices.cpu().numpy(), ref[1])


@pytest.mark.parametrize("n,budget_chunks", [(32768, 64), (4096, 31), (2048, 2), (5000, 1), (17, 31)])
def test_large_and_edge_selection_vs_oracle(dsb, cuda, n, budget_chunks):
    c = 32
    s = R.rng(n).random(n, dtype=np.float32)
    seq_len = n * c
    sel = dsb.selection.select_context_chunks(torch.from_numpy(s).to(cuda), seq_len, c, budget_chunks * c)
    ref = O.select_context_chunks(s, seq_len, c, budget_chunks * c)
    np.testing.assert_array_equal(sel.chunk_indices.cpu().numpy(), ref[0])
    np.testing.assert_array_equal(sel.token_indices.cpu().numpy(), ref[1])


def test_empty_sequence_and_uncommitted_rows(dsb, cuda):
    sel = dsb.selection.select_context_chunks(torch.empty(0, device=cuda), 0, 16, 64)
    assert sel.chunk_indices.numel() == 0 and sel.token_indices.numel() == 0
    parts = torch.rand((3, 2, 50), device=cuda)
    seq = torch.tensor([50 * 16, 0, 33], dtype=torch.int32, device=cuda)
    slots = torch.tensor([2, 0, -1], dtype=torch.int32, device=cuda)
    sel_chunks = torch.full((3, 4), 99, dtype=torch.int32, device=cuda)
    sel_count = torch.full((3,), -1, dtype=torch.int32, device=cuda)
    dsb.selection.select_rows(parts, seq, chunk_size=16, token_budget=64, normalize_heads=8,
                              row_slots=slots, sel_chunks=sel_chunks, sel_count=sel_count)
    counts = sel_count.cpu().tolist()
    assert counts == [0, -1, 4]  # slot 0: empty selection, slot 1: untouched, slot 2: 4 chunks
    s = parts[0].sum(0).cpu().numpy() / 16 / 8
    ref = O.select_context_chunks(s, 50 * 16, 16, 64)[0]
    assert sel_chunks[2].cpu().tolist() == ref.tolist()
    assert sel_chunks[1].cpu().tolist() == [99] * 4


@pytest.mark.parametrize("chunk", [2, 8, 64])
def test_device_plans_match_reference_exactly(dsb, cuda, chunk):
    """All 600 reference plans of the 200-trial sweep (tests/test_runtime.py:654-690)."""
    d = golden("plans")
    meta = d[f"c{chunk}_meta"]
    chunks, plans, idx = d[f"c{chunk}_chunks"], d[f"c{chunk}_plans"], d[f"c{chunk}_indices"]
    width = 5 + 8  # token_budget = 8 * chunk in the reference sweep
    cases = []
    co = po = 0
    for hb, he, _slot, nsel, nplan, _ in meta:
        sel = chunks[co:co + max(nsel, 0)]
        co += max(nsel, 0)
        cases.append((int(hb), int(he), int(nsel), sel, plans[po:po + nplan]))
        po += nplan
    for hb in sorted({c[0] for c in cases}):
        group = [c for c in cases if c[0] == hb]
        rows = len(group)
        sel_chunks = torch.zeros((rows, 8), dtype=torch.int32)
        sel_count = torch.tensor([c[2] for c in group], dtype=torch.int32)
        for r, c in enumerate(group):
            sel_chunks[r, : c[2] if c[2] > 0 else 0] = torch.from_numpy(c[3].astype(np.int32))
        committed = torch.tensor([c[1] + 1 for c in group], dtype=torch.int32)
        plan, hl = dsb.selection.build_history_plan(
            torch.arange(rows, dtype=torch.int32, device=cuda), committed.to(cuda),
            sel_chunks.to(cuda), sel_count.to(cuda), chunk_size=chunk, history_budget=hb,
            working_budget=8 * chunk)
        plan = plan.cpu().numpy()
        for r, c in enumerate(group):
            ref = c[4].copy()
            ref[0] = r  # the device rows use slot r
            np.testing.assert_array_equal(plan[r, : ref.size], ref)
            assert not plan[r, ref.size:].any()
            assert int(hl[r]) == ref[1]
            expanded = O.decode_history_plan(plan[r, : ref.size], chunk)
            assert all(0 <= t < c[1] for t in expanded)
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0
    del idx
