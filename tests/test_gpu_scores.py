"""Chunk-score retrieval kernels (rows A1/A2) against the reference and the oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import recipes as R
from conftest import golden
from oracle import diffspec_oracle as O

pytestmark = pytest.mark.gpu

_DT = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


def dev(a, device, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(device)
    return t.to(dtype) if dtype is not None else t


def no_flags(dsb, device):
    flag = dsb._lib.read_and_clear_error_flag(device)
    assert flag == 0, dsb._lib.describe_flag(flag)


@pytest.mark.parametrize("i", range(len(R.SCORE_CASES)))
def test_scores_match_reference_kernel_and_oracle(dsb, cuda, i):
    d = golden("scores")
    inp = R.scores_inputs(i)
    dt = _DT[inp["dtype"]]
    q, kc = dev(inp["query"], cuda, dt), dev(inp["key_cache"], cuda, dt)
    bt, seq = dev(inp["block_table"], cuda), dev(inp["lengths"], cuda)
    lse = dev(d[f"case{i}_lse"], cuda)
    got = dsb.kernels.paged_chunk_attention_scores(
        q, kc, lse, bt, seq, chunk_size=inp["chunk"], max_seq_len=inp["max_len"],
        scale=inp["scale"]).cpu().numpy()
    torch.cuda.synchronize()
    no_flags(dsb, cuda)
    # tolerance of the reference's own device test (tests/test_retrieval_npu.py:84)
    np.testing.assert_allclose(got, d[f"case{i}_ref_triton_scores"], rtol=1e-3, atol=1e-6)
    oracle = O.paged_chunk_attention_scores(inp["query"], inp["key_cache"], d[f"case{i}_lse"],
                                            inp["block_table"], inp["lengths"], inp["chunk"],
                                            inp["max_len"], inp["scale"])
    np.testing.assert_allclose(got, oracle, rtol=1e-4, atol=1e-7)
    assert np.isfinite(got).all()


@pytest.mark.parametrize("i", range(len(R.SCORE_CASES)))
def test_lse_free_scores_match_reference_dense(dsb, cuda, i):
    d = golden("scores")
    inp = R.scores_inputs(i)
    dt = _DT[inp["dtype"]]
    got = dsb.kernels.paged_chunk_attention_scores(
        dev(inp["query"], cuda, dt), dev(inp["key_cache"], cuda, dt), None,
        dev(inp["block_table"], cuda), dev(inp["lengths"], cuda), chunk_size=inp["chunk"],
        max_seq_len=inp["max_len"], scale=inp["scale"]).cpu().numpy()
    no_flags(dsb, cuda)
    for r, length in enumerate(inp["lengths"]):
        if length == 0:
            assert not got[r].any()
            continue
        ref = d[f"case{i}_ref_dense_nolse_row{r}"]
        np.testing.assert_allclose(got[r, : ref.size], ref, rtol=1e-3, atol=1e-7)
        assert not got[r, ref.size:].any()


def _random_paged(seed, b, length, hq, hk, d, bs, device, planted=0):
    g = R.rng(seed)
    pages = (length + bs - 1) // bs
    nblocks = b * pages + 5
    q = R.normal(g, (b, hq, d), "bf16")
    kc = R.normal(g, (nblocks, bs, hk, d), "bf16")
    table = g.permutation(nblocks)[: b * pages].reshape(b, pages).astype(np.int32)
    for r in range(b):
        for c in g.choice(length // 64 - 1, size=planted, replace=False):
            for t in range(64 * int(c), 64 * int(c) + 64):
                page, off = table[r][t // bs], t % bs
                kc[page, off] = R.round_to(
                    q[r].reshape(hk, hq // hk, d).mean(1) + 0.1 * g.standard_normal((hk, d)), "bf16")
    return q, kc, table


def test_head_partials_are_deterministic_and_shard_invariant(dsb, cuda):
    """The per-kv-head mass of a head shard equals the slice of the all-head
    result bit for bit: the property that makes selection identical at any
    number of head-sharded GPUs."""
    b, length, hq, hk, d, bs, c = 3, 5000, 32, 4, 128, 16, 64
    q, kc, table = _random_paged(11, b, length, hq, hk, d, bs, cuda)
    qd, kd = dev(q, cuda, torch.bfloat16), dev(kc, cuda, torch.bfloat16)
    bt = dev(table, cuda)
    seq = torch.tensor([length, 4097, 64], dtype=torch.int32, device=cuda)
    lse = torch.rand((b, hq), device=cuda) + 6.0
    kw = dict(chunk_size=c, max_seq_len=length, scale=d ** -0.5)
    full = dsb.kernels.paged_chunk_head_scores(qd, kd, lse, bt, seq, **kw)
    again = dsb.kernels.paged_chunk_head_scores(qd, kd, lse, bt, seq, **kw)
    assert torch.equal(full, again)
    for shards in (2, 4):
        per = hk // shards
        parts = []
        for s in range(shards):
            heads = slice(s * per, (s + 1) * per)
            qheads = slice(s * per * (hq // hk), (s + 1) * per * (hq // hk))
            parts.append(dsb.kernels.paged_chunk_head_scores(
                qd[:, qheads].contiguous(), kd[:, :, heads].contiguous(),
                lse[:, qheads].contiguous(), bt, seq, **kw))
        assert torch.equal(torch.cat(parts, dim=1), full)
    no_flags(dsb, cuda)


def test_full_length_scores_and_certified_selection(dsb, cuda):
    """One config-2 request (40960 tokens, 32/4 heads, chunk 64, 8 planted
    chunks): scores vs the fp64 oracle, and the top-k selection bit-exact
    wherever the fp64 boundary gap exceeds fp32 rounding."""
    b, length, hq, hk, d, bs, c, hb = 2, 40960, 32, 4, 128, 16, 64, 1984
    q, kc, table = _random_paged(12, b, length, hq, hk, d, bs, cuda, planted=8)
    seq_np = np.array([length, length - 3], dtype=np.int32)
    lse = R.dense_lse(dict(query=q, key_cache=kc, block_table=table, lengths=seq_np, hk=hk,
                           block_size=bs, scale=d ** -0.5))
    qd, kd, bt = dev(q, cuda, torch.bfloat16), dev(kc, cuda, torch.bfloat16), dev(table, cuda)
    seq, lse_d = dev(seq_np, cuda), dev(lse, cuda)
    parts = dsb.kernels.paged_chunk_head_scores(qd, kd, lse_d, bt, seq, chunk_size=c,
                                                max_seq_len=length, scale=d ** -0.5)
    scores = dsb.kernels.finalize_chunk_scores(parts, seq, chunk_size=c, total_query_heads=hq)
    oracle = O.paged_chunk_attention_scores(q, kc, lse, table, seq_np, c, length, d ** -0.5)
    np.testing.assert_allclose(scores.cpu().numpy(), oracle, rtol=1e-4, atol=1e-9)
    ci, ti, cs = dsb.selection.select_rows(parts, seq, chunk_size=c, token_budget=hb,
                                           normalize_heads=hq, with_outputs=True)
    gpu_scores = scores.cpu().numpy()
    for r in range(b):
        n = (int(seq_np[r]) + c - 1) // c
        same_input = O.select_context_chunks(gpu_scores[r, :n], int(seq_np[r]), c, hb)
        np.testing.assert_array_equal(ci[r].cpu().numpy(), same_input[0])
        got_tokens = ti[r].cpu().numpy()
        np.testing.assert_array_equal(got_tokens[: same_input[1].size], same_input[1])
        assert (got_tokens[same_input[1].size:] == -1).all()
        margin = O.selection_margin(oracle[r, :n], int(seq_np[r]), c, hb)
        if margin > 1e-5:  # fp32 rounding of these sums stays far below 1e-5
            np.testing.assert_array_equal(ci[r].cpu().numpy(),
                                          O.select_context_chunks(oracle[r, :n], int(seq_np[r]), c, hb)[0])
    no_flags(dsb, cuda)


def test_out_of_range_pages_and_query_rows_are_flagged_not_read(dsb, cuda):
    b, hq, hk, d, bs = 2, 8, 1, 128, 16
    q = torch.randn((b, hq, d), device=cuda).bfloat16()
    kc = torch.randn((4, bs, hk, d), device=cuda).bfloat16()
    bt = torch.tensor([[0, 1, 99], [2, 3, -1]], dtype=torch.int32, device=cuda)
    seq = torch.tensor([40, 20], dtype=torch.int32, device=cuda)
    lse = torch.zeros((b, hq), device=cuda)
    out = dsb.kernels.paged_chunk_head_scores(q, kc, lse, bt, seq, chunk_size=16, max_seq_len=40,
                                              scale=0.1)
    torch.cuda.synchronize()
    flag = dsb._lib.read_and_clear_error_flag(cuda)
    assert flag & 4  # block-table entry out of range
    assert torch.isfinite(out).all()
    qi = torch.tensor([0, 7], dtype=torch.int32, device=cuda)
    out = dsb.kernels.paged_chunk_head_scores(q, kc, lse, bt[:, :2], torch.tensor(
        [32, 32], dtype=torch.int32, device=cuda), chunk_size=16, max_seq_len=32, scale=0.1,
        query_index=qi)
    torch.cuda.synchronize()
    assert dsb._lib.read_and_clear_error_flag(cuda) & 2
    assert not out[1].any()
