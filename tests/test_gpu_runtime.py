"""DiffSpecDraftCache on the GPU: the retrieval hook against the reference's
own accept_target_queries, and a whole draft cycle against the oracle."""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest
import torch

import recipes as R
from conftest import close_bf16, golden
from oracle import diffspec_oracle as O

pytestmark = pytest.mark.gpu


def _cache(dsb, cuda, *, chunk, budget, depth, slots, max_len, hk, d, interval=1, table=None):
    settings = dsb.runtime.DiffSpecSettings(chunk, budget, interval, 4, depth, 0.7, False)
    if table is None:
        table = torch.from_numpy(R.round_to(R.cos_sin_table(budget, d), "bf16")).bfloat16()
    return dsb.runtime.DiffSpecDraftCache(
        settings, max_num_reqs=slots, max_model_len=max_len, num_kv_heads=hk, head_dim=d,
        target_num_layers=2, dtype=torch.bfloat16, device=cuda, cos_sin_cache=table,
        rotary_dim=d, is_neox_style=True)


def _tokens(chunks, length, chunk):
    if not chunks:
        return []
    out = [t for c in chunks[:-1] for t in range(c * chunk, (c + 1) * chunk)]
    return out + list(range(chunks[-1] * chunk, min(length, (chunks[-1] + 1) * chunk)))


@pytest.mark.parametrize("i", range(len(R.HOOK_CASES)))
def test_retrieval_hook_matches_reference(dsb, cuda, i):
    d = golden("hook")
    inp = R.hook_inputs(i)
    p = f"case{i}_"
    cache = _cache(dsb, cuda, chunk=R.HOOK_CHUNK, budget=R.HOOK_BUDGET, depth=3, slots=2,
                   max_len=256, hk=R.HOOK_HK, d=R.HOOK_D)
    assert cache.history_budget == int(d[p + "history_budget"])
    meta = SimpleNamespace(actual_seq_lengths_q=inp["query_ends"].tolist(),
                           seq_lens_list=inp["seq_lens"].tolist(),
                           block_tables=torch.from_numpy(inp["block_tables"]).to(cuda), num_prefills=0)
    cache.begin_target_forward(["a", "b"])
    cache.capture_target_attention(
        torch.from_numpy(inp["query"]).to(cuda).bfloat16(), torch.from_numpy(inp["lse"]).to(cuda),
        torch.from_numpy(inp["key_cache"]).to(cuda).bfloat16(), meta, R.HOOK_D ** -0.5)
    cache.accept_target_queries(torch.from_numpy(inp["counts"]).to(cuda), is_prefill=False)
    counts = cache.sel_count.cpu().tolist()
    chunks = cache.sel_chunks.cpu().numpy()
    _, r_len, r_slot = O.prepare_retrieval_rows(inp["query_ends"][:2], inp["seq_lens"][:2],
                                                inp["counts"], [0, 1])
    for slot in range(2):
        ref = d[p + f"ref_selected_slot{slot}"].tolist()
        if ref == [-2]:
            assert counts[slot] == -1
            continue
        got = _tokens(chunks[slot, : counts[slot]].tolist(), r_len[slot], R.HOOK_CHUNK)
        assert got == ref
    status = cache.retrieval_status()
    assert [status["retrieval_count"], status["retrieval_skipped_no_committed_tokens"]] == \
        d[p + "ref_status"].tolist()
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0


def test_retrieval_cadence_prefill_and_snapshot_counters(dsb, cuda):
    """tests/test_runtime.py:532-613 flow: prefill and interval skips, and no
    reuse of a stale snapshot."""
    cache = _cache(dsb, cuda, chunk=2, budget=8, depth=2, slots=2, max_len=8, hk=1, d=64,
                   interval=2)
    q = torch.randn((2, 2, 64), device=cuda).bfloat16()
    meta = SimpleNamespace(actual_seq_lengths_q=[1, 2], seq_lens_list=[6, 4],
                           block_tables=torch.zeros((2, 1), dtype=torch.int32, device=cuda),
                           num_prefills=0)
    kc = torch.randn((1, 8, 1, 64), device=cuda).bfloat16()
    cache.begin_target_forward(["r0", "r1"])
    cache.accept_target_queries(torch.ones(2, device=cuda), is_prefill=True)
    cache.capture_target_attention(q, torch.zeros((2, 2), device=cuda), kc, meta, 0.5)
    cache.accept_target_queries(torch.ones(2, device=cuda), is_prefill=True)
    cache.accept_target_queries(torch.ones(2, device=cuda), is_prefill=False)
    assert cache.sel_count.cpu().tolist() == [-1, -1]
    cache.accept_target_queries(torch.ones(2, dtype=torch.int64, device=cuda), is_prefill=False)
    s = cache.retrieval_status()
    assert (s["retrieval_skipped_prefill"], s["retrieval_skipped_interval"], s["retrieval_count"],
            s["selected_slots"]) == (1, 1, 1, 2)
    cache.begin_target_forward(["r1"])
    cache.accept_target_queries(torch.ones(1, device=cuda), is_prefill=cache.target_is_prefill)
    s = cache.retrieval_status()
    assert s["retrieval_skipped_no_snapshot"] == 2 and s["retrieval_count"] == 1


def test_full_draft_cycle_vs_oracle(dsb, cuda):
    """Retrieval -> plan -> rebuild -> 4 draft attention steps for 4 requests
    (config-2 head layout, shorter context), checked stage by stage."""
    b, length, hq, hk, d, bs, c, budget, depth = 4, 8192, 32, 4, 128, 16, 64, 1024, 4
    g = R.rng(321)
    pages = length // bs
    key_cache = R.normal(g, (b * pages, bs, hk, d), "bf16")
    table = g.permutation(b * pages).reshape(b, pages).astype(np.int32)
    # target verify pass: 5 query tokens per request (root + 4 drafts)
    query = R.normal(g, (5 * b, hq, d), "bf16")
    seq = np.array([length - 10, length - 200, length - 1000, 3000], np.int32)
    counts = np.array([3, 5, 1, 2], np.int64)
    ends = np.arange(1, b + 1, dtype=np.int32) * 5
    q_idx, r_len, _ = O.prepare_retrieval_rows(ends, seq, counts, list(range(b)))
    lse_rows = R.dense_lse(dict(query=query[q_idx], key_cache=key_cache, block_table=table,
                                lengths=np.array(r_len, np.int32), hk=hk, block_size=bs,
                                scale=d ** -0.5))
    lse = np.zeros((5 * b, hq), np.float32)
    lse[q_idx] = lse_rows
    cos_sin = R.round_to(R.cos_sin_table(budget, d), "bf16")
    cache = _cache(dsb, cuda, chunk=c, budget=budget, depth=depth, slots=6, max_len=length, hk=hk,
                   d=d, table=torch.from_numpy(cos_sin).bfloat16())
    raw_k = R.normal(g, (6, length, hk, d), "bf16")
    raw_v = R.normal(g, (6, length, hk, d), "bf16")
    cache.raw_key.copy_(torch.from_numpy(raw_k))
    cache.raw_value.copy_(torch.from_numpy(raw_v))
    ids = ["w", "x", "y", "z"]
    cache.begin_target_forward(ids)
    meta = SimpleNamespace(actual_seq_lengths_q=ends.tolist(), seq_lens_list=seq.tolist(),
                           block_tables=torch.from_numpy(table).to(cuda), num_prefills=0)
    cache.capture_target_attention(torch.from_numpy(query).to(cuda).bfloat16(),
                                   torch.from_numpy(lse).to(cuda),
                                   torch.from_numpy(key_cache).to(cuda).bfloat16(), meta, d ** -0.5)
    cache.accept_target_queries(torch.from_numpy(counts).to(cuda), is_prefill=False)
    hb = cache.history_budget
    oracle_scores = O.paged_chunk_attention_scores(query[q_idx], key_cache, lse_rows, table,
                                                   np.array(r_len), c, max(r_len), d ** -0.5)
    sel = {}
    for r in range(b):
        n = (r_len[r] + c - 1) // c
        assert O.selection_margin(oracle_scores[r, :n], r_len[r], c, hb) > 1e-5
        sel[r] = O.select_context_chunks(oracle_scores[r, :n], r_len[r], c, hb)[0].tolist()
        assert cache.sel_chunks[r, : cache.sel_count[r]].cpu().tolist() == sel[r]
    # draft cycle: committed root = last accepted target position
    committed = (seq - 5 + counts).tolist()
    cache.begin_cycle(ids)
    hl = cache.rebuild(committed).cpu().tolist()
    wk_o = np.zeros((6, hk, budget, d), np.float32)
    wv_o = np.zeros_like(wk_o)
    plans = np.zeros((b, 5 + budget // c), np.int64)
    for r in range(b):
        pl = O.history_plan(r, sel[r], committed[r] - 1, c, hb)
        plans[r, : len(pl)] = pl
        assert hl[r] == pl[1]
    O.rebuild_compact_kv_from_plan(raw_k, raw_v, wk_o, wv_o, plans, cos_sin, c, hb, d, True, "bf16")
    for r in range(b):
        h = hl[r]
        np.testing.assert_array_equal(cache.working_key[r, :, :h].float().cpu().numpy(), wk_o[r, :, :h])
        np.testing.assert_array_equal(cache.working_value[r, :, :h].float().cpu().numpy(), wv_o[r, :, :h])
    for step in range(depth):
        qs = R.normal(g, (8, hq, d), "bf16")
        ks = R.normal(g, (8, hk, d), "bf16")
        vs = R.normal(g, (8, hk, d), "bf16")
        out = torch.empty((8, hq, d), device=cuda).bfloat16()
        cache.forward_attention(torch.from_numpy(qs).to(cuda).bfloat16(),
                                torch.from_numpy(ks).to(cuda).bfloat16(),
                                torch.from_numpy(vs).to(cuda).bfloat16(), d ** -0.5, out)
        ref = O.draft_decode_attention(qs[:b], ks[:b], vs[:b], wk_o, wv_o, list(range(b)),
                                       [h + step for h in hl], d ** -0.5, out_rows=8, dtype=None)
        close_bf16(out.float().cpu().numpy(), ref)
    with pytest.raises(RuntimeError, match="exhausted"):
        for _ in range(budget):
            cache.forward_attention(torch.from_numpy(qs).to(cuda).bfloat16(),
                                    torch.from_numpy(ks).to(cuda).bfloat16(),
                                    torch.from_numpy(vs).to(cuda).bfloat16(), d ** -0.5, out)
    torch.cuda.synchronize()
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0
