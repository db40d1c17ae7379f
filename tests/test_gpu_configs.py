"""BASELINE config 2's retrieval batch and configs 3 and 4 at their full sizes (rows A1-A8, e).

At these sizes the oracle cannot score every row, so the tests combine
size-independent properties over all rows with oracle checks of sampled
rows: config 4 (32 requests x 131072 tokens, 64 / 8 heads) checks that the
head-sharded retrieval is bit-identical at 1, 2, 4 and 8 shards and that the
planted chunks are found; config 3 (64 ragged requests up to 131072 tokens,
reordered slots, rows with nothing committed, graph padding) runs the whole
draft cycle through DiffSpecDraftCache and checks every stage."""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest
import torch

import recipes as R
from conftest import close_bf16
from oracle import diffspec_oracle as O

pytestmark = pytest.mark.gpu


def _paged_keys(gen, lengths, hk, d, bs, device):
    """Device paged K for ragged rows in a shuffled block table."""
    pages = [(int(n) + bs - 1) // bs for n in lengths]
    width = max(pages)
    nblocks = sum(pages) + 3
    kc = torch.randn((nblocks, bs, hk, d), generator=gen, device=device).to(torch.bfloat16)
    perm = torch.randperm(nblocks, generator=gen, device=device).to(torch.int32)
    table = torch.zeros((len(lengths), width), dtype=torch.int32, device=device)
    off = 0
    for r, p in enumerate(pages):
        table[r, :p] = perm[off:off + p]
        off += p
    return kc, table


def _row_to_host(kc, table, r, length, bs):
    """One row's pages as a host paged cache with an identity block table."""
    p = (length + bs - 1) // bs
    keys = kc[table[r, :p].long()].float().cpu().numpy()
    return keys, np.arange(p, dtype=np.int32)[None]


def test_config4_retrieval_identical_at_any_head_shard_count(dsb, cuda):
    """Config 4: per-kv-head mass of every shard layout (8 kv heads over 1,
    2, 4, 8 GPUs, simulated by head slices in global head order) is the
    same bits, so the selected chunks are identical; planted chunks are
    selected; one row is checked against the oracle."""
    b, length, hq, hk, d, bs, c, w = 32, 131072, 64, 8, 128, 16, 64, 4096
    hb = (w - 4 - 1) // c * c
    gen = torch.Generator(device=cuda)
    gen.manual_seed(4)
    kc, table = _paged_keys(gen, [length] * b, hk, d, bs, cuda)
    q = torch.randn((b, hq, d), generator=gen, device=cuda).to(torch.bfloat16)
    planted = []
    for r in range(b):  # 4 planted chunks per row: keys = group-mean query + noise
        chunks = torch.randperm(length // c - 1, generator=gen, device=cuda)[:4]
        planted.append(sorted(chunks.tolist()))
        tok = (chunks[:, None] * c + torch.arange(c, device=cuda)).reshape(-1)
        target = q[r].float().view(hk, hq // hk, d).mean(1)
        noise = 0.1 * torch.randn((tok.numel(), hk, d), generator=gen, device=cuda)
        kc[table[r, tok // bs].long(), tok % bs] = (target + noise).to(torch.bfloat16)
    seq = torch.full((b,), length - 2, dtype=torch.int32, device=cuda)
    lse = torch.rand((b, hq), generator=gen, device=cuda) + 9.0
    kw = dict(chunk_size=c, max_seq_len=length, scale=d ** -0.5)
    full = dsb.kernels.paged_chunk_head_scores(q, kc, lse, table, seq, **kw)
    sel_full = dsb.selection.select_rows(full, seq, chunk_size=c, token_budget=hb,
                                         normalize_heads=hq, with_outputs=True)[0]
    group = hq // hk
    for shards in (2, 4, 8):
        per = hk // shards
        parts = []
        for s in range(shards):
            kv = slice(s * per, (s + 1) * per)
            qh = slice(s * per * group, (s + 1) * per * group)
            k_shard = kc[:, :, kv].contiguous()
            parts.append(dsb.kernels.paged_chunk_head_scores(
                q[:, qh].contiguous(), k_shard, lse[:, qh].contiguous(), table, seq, **kw))
            del k_shard
        gathered = torch.cat(parts, dim=1)
        assert torch.equal(gathered, full)
        sel = dsb.selection.select_rows(gathered, seq, chunk_size=c, token_budget=hb,
                                        normalize_heads=hq, with_outputs=True)[0]
        assert torch.equal(sel, sel_full)
        # the all-gather's rank-major layout, read in place by the selection
        stacked = torch.stack(parts, dim=0)
        sel = dsb.selection.select_rows(stacked, seq, chunk_size=c, token_budget=hb,
                                        normalize_heads=hq, with_outputs=True)[0]
        assert torch.equal(sel, sel_full)
    sel_host = sel_full.cpu().numpy()
    for r in range(b):
        assert set(planted[r]) <= set(sel_host[r].tolist())
    # one row against the oracle
    keys, t_row = _row_to_host(kc, table, 0, length, bs)
    ref = O.paged_chunk_attention_scores(q[:1].float().cpu().numpy(), keys, lse[:1].cpu().numpy(),
                                         t_row, np.array([length - 2]), c, length, d ** -0.5)
    got = dsb.kernels.finalize_chunk_scores(full[:1], seq[:1], chunk_size=c, total_query_heads=hq)
    np.testing.assert_allclose(got.cpu().numpy(), ref, rtol=1e-3, atol=1e-9)
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0


def test_config2_batch_selection_and_plans(dsb, cuda):
    """Config 2's whole retrieval batch as the bench runs it: 16 requests x
    40960 tokens (3 rejected, 40957 scored), 32 / 4 heads, chunk 64, budget
    2048 (history 1984), rolling window 256, 8 planted chunks per request,
    the LSE computed on the device (softmax_lse=None).  Every row is scored
    by the fp64 oracle: the GPU scores match it, the selection equals the
    oracle's selection of the GPU's own scores on every row and the oracle's
    selection of its fp64 scores wherever the boundary gap exceeds fp32
    rounding, the planted chunks are selected, and the plans of four cycles
    (two accepted tokens each) equal the oracle's plan rows bit for bit."""
    b, length, hq, hk, d, bs, c, hb, win = 16, 40960, 32, 4, 128, 16, 64, 1984, 256
    seq_len = length - 3
    n = (seq_len + c - 1) // c
    gen = torch.Generator(device=cuda)
    gen.manual_seed(22)
    kc, table = _paged_keys(gen, [length] * b, hk, d, bs, cuda)
    q = torch.randn((b, hq, d), generator=gen, device=cuda).to(torch.bfloat16)
    planted = []
    for r in range(b):  # keys = group-mean query + noise
        chunks = torch.randperm(n - win // c, generator=gen, device=cuda)[:8]
        planted.append(sorted(chunks.tolist()))
        tok = (chunks[:, None] * c + torch.arange(c, device=cuda)).reshape(-1)
        target = q[r].float().view(hk, hq // hk, d).mean(1)
        noise = 0.1 * torch.randn((tok.numel(), hk, d), generator=gen, device=cuda)
        kc[table[r, tok // bs].long(), tok % bs] = (target + noise).to(torch.bfloat16)
    seq = torch.full((b,), seq_len, dtype=torch.int32, device=cuda)
    kw = dict(chunk_size=c, max_seq_len=length, scale=d ** -0.5)
    parts = dsb.kernels.paged_chunk_head_scores(q, kc, None, table, seq, **kw)
    scores = dsb.kernels.finalize_chunk_scores(parts, seq, chunk_size=c,
                                               total_query_heads=hq).cpu().numpy()
    slots = torch.arange(b, dtype=torch.int32, device=cuda)
    sel_chunks = torch.zeros((b, hb // c), dtype=torch.int32, device=cuda)
    sel_count = torch.full((b,), -1, dtype=torch.int32, device=cuda)
    ci = dsb.selection.select_rows(parts, seq, chunk_size=c, token_budget=hb, normalize_heads=hq,
                                   row_slots=slots, sel_chunks=sel_chunks, sel_count=sel_count,
                                   with_outputs=True, recent_window=win)[0].cpu().numpy()
    certified = 0
    for r in range(b):
        keys, t_row = _row_to_host(kc, table, r, length, bs)
        oracle = O.paged_chunk_attention_scores(q[r:r + 1].float().cpu().numpy(), keys, None, t_row,
                                                np.array([seq_len]), c, length, d ** -0.5)[0]
        np.testing.assert_allclose(scores[r, :n], oracle[:n], rtol=1e-3, atol=1e-9)
        own = O.select_context_chunks(scores[r, :n], seq_len, c, hb, recent_window=win)[0]
        got = ci[r][ci[r] >= 0]
        np.testing.assert_array_equal(got, own)
        if O.selection_margin(oracle[:n], seq_len, c, hb, recent_window=win) > 1e-5:
            certified += 1
            np.testing.assert_array_equal(
                got, O.select_context_chunks(oracle[:n], seq_len, c, hb, recent_window=win)[0])
        assert set(planted[r]) <= set(got.tolist())
    assert certified >= b // 2  # most rows have a clear top-k boundary
    chosen = [sel_chunks[r, : int(sel_count[r])].cpu().tolist() for r in range(b)]
    for cycle in range(4):
        committed = torch.full((b,), seq_len + 1 + 2 * cycle, dtype=torch.int32, device=cuda)
        plan, hl = dsb.selection.build_history_plan(
            slots, committed, sel_chunks, sel_count, chunk_size=c, history_budget=hb,
            working_budget=2048, recent_window=win)
        plan = plan.cpu().numpy()
        for r in range(b):
            expect = O.history_plan(r, chosen[r], int(committed[r]) - 1, c, hb, recent_window=win)
            assert plan[r, : len(expect)].tolist() == expect
            assert (plan[r, len(expect):] == 0).all()
            assert int(hl[r]) == expect[1]
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0


def _cache(dsb, cuda, *, chunk, budget, depth, slots, max_len, hk, d, table):
    settings = dsb.runtime.DiffSpecSettings(chunk, budget, 1, 4, depth, 0.7, False)
    return dsb.runtime.DiffSpecDraftCache(
        settings, max_num_reqs=slots, max_model_len=max_len, num_kv_heads=hk, head_dim=d,
        target_num_layers=2, dtype=torch.bfloat16, device=cuda, cos_sin_cache=table,
        rotary_dim=d, is_neox_style=True)


def test_config3_ragged_draft_cycle(dsb, cuda):
    """Config 3: 64 requests, lengths ~ U[2048, 131072], chunk 32, budget
    2048, rejected suffix ~ U[0, 4], 8 requests with nothing committed,
    reordered slots, 8 graph-padding rows.  Retrieval is checked against the
    oracle on sampled rows (where the selection margin exceeds fp32
    rounding), plans and rebuilt rows and attention on every row."""
    b, hq, hk, d, bs, c, budget, depth, pad = 64, 32, 4, 128, 16, 32, 2048, 4, 8
    g = R.rng(3003)
    lengths = g.integers(2048, 131072 + 1, size=b).astype(np.int32)
    counts = g.integers(1, 6, size=b).astype(np.int64)  # accepted tokens of 5 verified
    counts[g.choice(b, size=8, replace=False)] = 0        # nothing committed
    gen = torch.Generator(device=cuda)
    gen.manual_seed(3)
    kc, table = _paged_keys(gen, lengths, hk, d, bs, cuda)
    query = torch.randn((5 * b, hq, d), generator=gen, device=cuda).to(torch.bfloat16)
    lse = torch.rand((5 * b, hq), generator=gen, device=cuda) + 10.0
    cos_sin = torch.from_numpy(R.round_to(R.cos_sin_table(budget, d), "bf16")).to(cuda).bfloat16()
    max_len = int(lengths.max()) + 8
    cache = _cache(dsb, cuda, chunk=c, budget=budget, depth=depth, slots=b, max_len=max_len, hk=hk,
                   d=d, table=cos_sin)
    cache.raw_key.normal_(generator=gen)
    cache.raw_value.normal_(generator=gen)
    ids = [f"r{i}" for i in range(b)]
    cache.set_active_requests(ids)              # slots 0..63 in id order
    order = g.permutation(b)
    ids = [ids[i] for i in order]                # same requests, reordered rows
    ends = (np.arange(1, b + 1) * 5).astype(np.int32)
    seq = lengths[order]
    cnt = counts[order]
    cache.begin_target_forward(ids)
    slots = cache.active_slots()
    assert slots == order.tolist()
    meta = SimpleNamespace(actual_seq_lengths_q=ends.tolist(), seq_lens_list=seq.tolist(),
                           block_tables=table[torch.from_numpy(order).to(cuda)], num_prefills=0)
    cache.capture_target_attention(query, lse, kc, meta, d ** -0.5)
    cache.accept_target_queries(torch.from_numpy(cnt).to(cuda), is_prefill=False)
    q_idx, r_len, r_slot = O.prepare_retrieval_rows(ends, seq, cnt, slots)
    hb = cache.history_budget
    sel_count = cache.sel_count.cpu().numpy()
    sel_chunks = cache.sel_chunks.cpu().numpy()
    # rows with nothing committed keep "no selection"
    for r in range(b):
        if r_slot[r] < 0:
            assert sel_count[slots[r]] == -1
    # sampled rows against the oracle: shortest, longest and three others
    live = [r for r in range(b) if r_slot[r] >= 0]
    sample = sorted({min(live, key=lambda r: r_len[r]), max(live, key=lambda r: r_len[r]),
                     *g.choice(live, size=3, replace=False).tolist()})
    tbl = table[torch.from_numpy(order).to(cuda)]
    checked = 0
    for r in sample:
        keys, t_row = _row_to_host(kc, tbl, r, r_len[r], bs)
        sc = O.paged_chunk_attention_scores(
            query[q_idx[r]:q_idx[r] + 1].float().cpu().numpy(), keys,
            lse[q_idx[r]:q_idx[r] + 1].cpu().numpy(), t_row, np.array([r_len[r]]), c, r_len[r],
            d ** -0.5)[0]
        n = (r_len[r] + c - 1) // c
        if O.selection_margin(sc[:n], r_len[r], c, hb) <= 1e-5:
            continue
        ref = O.select_context_chunks(sc[:n], r_len[r], c, hb)[0]
        s = slots[r]
        np.testing.assert_array_equal(sel_chunks[s, : sel_count[s]], ref)
        checked += 1
    assert checked >= 3
    # draft cycle: every row's plan, working cache and four attention steps
    committed = (seq - 5 + cnt).tolist()
    cache.begin_cycle(ids)
    hl = cache.rebuild(committed).cpu().tolist()
    plan = cache._plan[:b].cpu().numpy()
    for r in range(b):
        s = slots[r]
        chunks = None if sel_count[s] < 0 else sel_chunks[s, : sel_count[s]].tolist()
        ref_plan = O.history_plan(s, chunks, committed[r] - 1, c, hb)
        np.testing.assert_array_equal(plan[r, : len(ref_plan)], ref_plan)
        assert not plan[r, len(ref_plan):].any()
        assert hl[r] == ref_plan[1]
        pos = torch.tensor(O.decode_history_plan(ref_plan, c), dtype=torch.long, device=cuda)
        src_k = cache.raw_key[s, pos].float().cpu().numpy()          # [h, hk, d]
        src_v = cache.raw_value[s, pos].float().cpu().numpy()
        cs = cos_sin[: hl[r]].float().cpu().numpy()
        exp_k = O.round_to(np.stack([O.rope_rotate(src_k[p], cs[p], d, True)
                                     for p in range(hl[r])]), "bf16") if hl[r] else src_k
        got_k = cache.working_key[s, :, : hl[r]].float().cpu().numpy().transpose(1, 0, 2)
        got_v = cache.working_value[s, :, : hl[r]].float().cpu().numpy().transpose(1, 0, 2)
        np.testing.assert_array_equal(got_k, exp_k)
        np.testing.assert_array_equal(got_v, src_v)
    wk = cache.working_key.float().cpu().numpy()
    wv = cache.working_value.float().cpu().numpy()
    for step in range(depth):
        qs = torch.randn((b + pad, hq, d), generator=gen, device=cuda).to(torch.bfloat16)
        ks = torch.randn((b + pad, hk, d), generator=gen, device=cuda).to(torch.bfloat16)
        vs = torch.randn((b + pad, hk, d), generator=gen, device=cuda).to(torch.bfloat16)
        out = torch.full((b + pad, hq, d), float("nan"), device=cuda).to(torch.bfloat16)
        cache.forward_attention(qs, ks, vs, d ** -0.5, out)
        for r in range(b):  # the oracle's working cache takes this step's token too
            wk[slots[r], :, hl[r] + step] = ks[r].float().cpu().numpy()
            wv[slots[r], :, hl[r] + step] = vs[r].float().cpu().numpy()
        ref = O.draft_decode_attention(qs[:b].float().cpu().numpy(), ks[:b].float().cpu().numpy(),
                                       vs[:b].float().cpu().numpy(), wk, wv, slots,
                                       [h + step for h in hl], d ** -0.5, out_rows=b + pad,
                                       dtype=None)
        got = out.float().cpu().numpy()
        close_bf16(got, ref)
        assert not got[b:].any()  # graph-padding rows are zero
    torch.cuda.synchronize()
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0
