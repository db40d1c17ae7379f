"""Known-answer vectors of the reference's own tests (tests/test_runtime.py),
restated on the oracle's functions."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import diffspec_oracle as O


def test_select_reserves_partial_tail():  # tests/test_runtime.py:301-310
    ci, ti, _ = O.select_context_chunks(np.array([0.1, 0.9, 0.8, 0.7, 0.01]), 18, 4, 12)
    assert ci.tolist() == [1, 2, 4]
    assert ti.tolist() == [4, 5, 6, 7, 8, 9, 10, 11, 16, 17]


def test_tp_retrieval_pools_all_target_heads():  # tests/test_runtime.py:41-69
    # two TP ranks' scores summed then divided by the TP size; chunk 2,
    # budget 8, depth 1 -> history budget 6 -> three chunks kept
    scores = (np.array([0., 100., 0., 0., 0.]) + np.array([0., 0., 0., 400., 0.])) / 2
    hb = O.history_budget(8, 1, 2)
    _, ti, _ = O.select_context_chunks(scores, 10, 2, hb)
    assert ti.tolist() == [2, 3, 6, 7, 8, 9]


def test_retrieval_uses_decode_queries():  # tests/test_runtime.py:532-613
    hb = O.history_budget(8, 2, 2)
    _, t0, _ = O.select_context_chunks(np.array([0.9, 0.1, 0.2]), 6, 2, hb)
    _, t1, _ = O.select_context_chunks(np.array([0.1, 0.9, 0.0])[:2], 4, 2, hb)  # first n chunks
    assert t0.tolist() == [0, 1, 4, 5] and t1.tolist() == [0, 1, 2, 3]


def test_rolling_tail_excludes_root():  # tests/test_runtime.py:616-634
    hb = O.history_budget(8, 2, 2)
    assert O.history_indices([0, 1, 4, 5], 5, 2, hb).tolist() == [0, 1, 3, 4]
    assert O.history_indices([0, 1, 4, 5], 9, 2, hb).tolist() == [0, 1, 7, 8]


@pytest.mark.parametrize("selected,history_end,expected", [  # tests/test_runtime.py:781-803
    (list(range(65)), 64, list(range(64))),
    (list(range(70)), 64, list(range(64))),
    (list(range(32)) + list(range(96, 128)), 127, list(range(32)) + list(range(95, 127))),
    (list(range(12)), 11, list(range(11))),
])
def test_unique_committed_history(selected, history_end, expected):
    hb = O.history_budget(128, 3, 32)
    assert O.history_indices(selected, history_end, 32, hb).tolist() == expected


@pytest.mark.parametrize("history_end", [0, 5, 7, 9, 13, 15])
def test_plan_matches_indices(history_end):  # tests/test_runtime.py:637-651
    hb = O.history_budget(8, 2, 2)
    for tokens, chunks in ((None, None), ([], []), ([0, 1, 4, 5], [0, 2]), ([2, 3, 8, 9], [1, 4])):
        expected = O.history_indices(tokens, history_end, 2, hb).tolist()
        plan = O.history_plan(0, chunks, history_end, 2, hb)
        assert O.decode_history_plan(plan, 2) == expected
        assert len(expected) <= hb and all(t < history_end for t in expected)


def test_dense_scores_vs_softmax():  # tests/test_runtime.py:270-298
    rng = np.random.default_rng(7)
    q = rng.standard_normal((4, 8))
    k = rng.standard_normal((11, 2, 8))
    scale = 8 ** -0.5
    got = O.chunk_attention_scores(q, k, 4, scale=scale)
    logits = np.einsum("hd,thd->ht", q, np.repeat(k, 2, axis=1)) * scale
    w = np.exp(logits - logits.max(1, keepdims=True))
    w /= w.sum(1, keepdims=True)
    np.testing.assert_allclose(got, [w[:, :4].mean(), w[:, 4:8].mean(), w[:, 8:].mean()], rtol=1e-12)
    lse = np.log(np.exp(logits).sum(1))
    np.testing.assert_allclose(O.chunk_attention_scores(q, k, 4, lse, scale), got, rtol=1e-12)


def test_cpu_draft_attention_vs_dense():  # tests/test_runtime.py:405-445
    wk = np.zeros((1, 1, 8, 2))
    wv = np.zeros((1, 1, 8, 2))
    wk[0, 0, :2] = [[1.0, 0.0], [0.0, 1.0]]
    wv[0, 0, :2] = [[2.0, 0.0], [0.0, 4.0]]
    q = np.array([[[1.0, 1.0], [1.0, -1.0]]])
    out = O.draft_decode_attention(q, np.array([[[1.0, 1.0]]]), np.array([[[6.0, 8.0]]]), wk, wv,
                                   [0], [2], 2 ** -0.5, dtype=None)
    keys = np.repeat(wk[0, :, :3], 2, axis=0)
    vals = np.repeat(wv[0, :, :3], 2, axis=0)
    logits = np.einsum("hd,hsd->hs", q[0], keys) * 2 ** -0.5
    p = np.exp(logits) / np.exp(logits).sum(1, keepdims=True)
    np.testing.assert_allclose(out[0], np.einsum("hs,hsd->hd", p, vals))


def test_committed_query_pick():  # tests/test_runtime.py:72-142 semantics
    q, r_len, slots = O.prepare_retrieval_rows([4, 8], [10, 12], [1, 2], [0, 1])
    assert q == [0, 5] and r_len == [7, 10] and slots == [0, 1]
    q, r_len, slots = O.prepare_retrieval_rows([4, 8], [10, 12], [0, 2], [0, 1])
    assert r_len == [0, 10] and slots == [-1, 1]
