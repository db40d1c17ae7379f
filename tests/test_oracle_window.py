"""The oracle's rolling-recent-window mode (no reference counterpart; the
reference's rolling tail is one chunk, diffspec/runtime.py:1657-1659,
1719-1720).  A window of one chunk must reproduce the reference's fixtures
exactly; longer windows must keep the mode's invariants: the tail is the
last min(window, history_end, budget) tokens, the prefix never overlaps it,
the plan row expands to the _history_indices restatement, and the ranked
chunks are the top-scoring ones that lie before the window."""

from __future__ import annotations

import numpy as np
import pytest

import recipes as R
from conftest import golden
from oracle import diffspec_oracle as O


def test_one_chunk_window_is_the_reference_selection():
    d = golden("select")
    for i, (seq_len, c, budget) in enumerate(R.select_cases()):
        n = (seq_len + c - 1) // c
        ci, ti, _ = O.select_context_chunks(R.select_scores(i, n), seq_len, c, budget,
                                            recent_window=c)
        np.testing.assert_array_equal(ci, d[f"case{i}_chunk_indices"])
        np.testing.assert_array_equal(ti, d[f"case{i}_token_indices"])


@pytest.mark.parametrize("chunk", [2, 8, 64])
def test_one_chunk_window_is_the_reference_plan(chunk):
    d = golden("plans")
    chunks, plans = d[f"c{chunk}_chunks"], d[f"c{chunk}_plans"]
    co = po = 0
    for hb, he, slot, nsel, nplan, _ in d[f"c{chunk}_meta"]:
        sel = None if nsel < 0 else chunks[co:co + nsel].tolist()
        co += max(nsel, 0)
        row = O.history_plan(int(slot), sel, int(he), chunk, int(hb), recent_window=chunk)
        np.testing.assert_array_equal(row, plans[po:po + nplan])
        po += nplan


@pytest.mark.parametrize("c,budget,window", [(32, 480, 128), (64, 1984, 256), (16, 256, 96)])
def test_window_selection_ranks_only_chunks_before_the_window(c, budget, window):
    g = R.rng(window + c)
    wc, s_cap = window // c, budget // c
    for trial in range(60):
        n = int(g.integers(s_cap + 1, 40 * s_cap))
        seq_len = n * c - int(g.integers(0, c))
        s = (g.integers(0, 20, n) / 4).astype(np.float32)
        ci, ti, cs = O.select_context_chunks(s, seq_len, c, budget, recent_window=window)
        ranked = ci[:-1]
        assert ci[-1] == n - 1 and ranked.size == s_cap - wc
        assert (np.diff(ci) > 0).all() and (ranked < n - wc).all()
        rest = np.setdiff1d(np.arange(n - wc), ranked)
        if rest.size:
            # top-k: no unselected candidate outranks a selected one; ties
            # go to the lower index
            worst = min(s[ranked].min(), np.inf)
            assert s[rest].max() <= worst
            tied = rest[s[rest] == worst]
            assert tied.size == 0 or tied.min() > ranked[s[ranked] == worst].max()
        np.testing.assert_array_equal(cs, s[ci])
        assert ti[-1] == seq_len - 1


@pytest.mark.parametrize("c,hb,window", [(32, 480, 128), (64, 1984, 256), (8, 64, 8), (16, 128, 128)])
def test_window_plans_expand_to_the_history_indices(c, hb, window):
    g = R.rng(hb * 3 + window)
    for trial in range(300):
        he = int(g.integers(0, 30 * hb))
        n = max(1, (he + 1 + c - 1) // c)
        if trial % 11 == 0:
            sel = None
        else:
            k = int(g.integers(0, min(n, hb // c) + 1))
            sel = sorted(g.choice(n, k, replace=False).tolist()) if k else []
        row = O.history_plan(0, sel, he, c, hb, recent_window=window)
        tokens = None if sel is None else np.array(
            [t for ch in sel for t in range(ch * c, ch * c + c)], np.int64)
        idx = O.history_indices(tokens, he, c, hb, recent_window=window)
        assert O.decode_history_plan(row, c) == idx.tolist()
        assert row[1] == idx.size <= hb
        assert len(set(idx.tolist())) == idx.size and (idx < max(he, 1)).all()
        if sel is not None:
            tail = min(he, window, hb)
            assert idx[idx.size - tail:].tolist() == list(range(he - tail, he))
            assert (idx[: idx.size - tail] < he - tail).all()


def test_window_validation():
    with pytest.raises(ValueError, match="recent_window"):
        O.select_context_chunks(np.zeros(40, np.float32), 40 * 16, 16, 256, recent_window=24)
    with pytest.raises(ValueError, match="recent_window"):
        O.select_context_chunks(np.zeros(40, np.float32), 40 * 16, 16, 256, recent_window=272)
    with pytest.raises(ValueError, match="recent_window"):
        O.select_context_chunks(np.zeros(40, np.float32), 40 * 16, 16, 256, recent_window=8)


def test_window_rejections_in_the_python_layer(dsb):
    """The package validates the window before touching a device."""
    import torch

    with pytest.raises(ValueError, match="recent_window"):
        dsb.selection.select_context_chunks(torch.zeros(40), 40 * 16, 16, 256, recent_window=24)
    settings = dsb.runtime.DiffSpecSettings(32, 512, 1, 4, 4, 0.7, False)
    with pytest.raises(ValueError, match="recent_window"):
        dsb.runtime.DiffSpecDraftCache(settings, max_num_reqs=1, max_model_len=64, num_kv_heads=1,
                                       head_dim=64, target_num_layers=1, dtype=torch.bfloat16,
                                       device="cpu", cos_sin_cache=torch.zeros(512, 64),
                                       recent_window=500)
