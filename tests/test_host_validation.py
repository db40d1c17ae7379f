"""Host-side validation mirrors the reference's ValueError conditions, and
CPU tensors are refused (there is no CPU fallback)."""

from __future__ import annotations

import pytest
import torch


def test_scores_validation(dsb):
    k = dsb.kernels
    q = torch.zeros((2, 8, 64), dtype=torch.bfloat16)
    kc = torch.zeros((4, 16, 2, 64), dtype=torch.bfloat16)
    bt = torch.zeros((2, 4), dtype=torch.int32)
    seq = torch.tensor([10, 20], dtype=torch.int32)
    lse = torch.zeros((2, 8))
    kw = dict(chunk_size=16, max_seq_len=20, scale=0.1)
    with pytest.raises(ValueError, match="query must have shape"):
        k.paged_chunk_attention_scores(q[0], kc, lse, bt, seq, **kw)
    with pytest.raises(ValueError, match="key_cache must have shape"):
        k.paged_chunk_attention_scores(q, kc[0], lse, bt, seq, **kw)
    with pytest.raises(ValueError, match="head dimensions must match"):
        k.paged_chunk_attention_scores(q, kc[..., :32], lse, bt, seq, **kw)
    with pytest.raises(ValueError, match="divisible by KV heads"):
        k.paged_chunk_attention_scores(q[:, :7], kc, lse[:, :7], bt, seq, **kw)
    with pytest.raises(ValueError, match="one value per query head"):
        k.paged_chunk_attention_scores(q, kc, lse[:, :4], bt, seq, **kw)
    with pytest.raises(ValueError, match="need CUDA tensors"):
        k.paged_chunk_attention_scores(q, kc, lse, bt, seq, **kw)


def test_rebuild_validation(dsb):
    f = dsb.compact_kv.rebuild_compact_kv_from_plan
    raw = torch.zeros((2, 32, 1, 64), dtype=torch.bfloat16)
    work = torch.zeros((2, 1, 16, 64), dtype=torch.bfloat16)
    plan = torch.zeros((2, 5 + 16 // 8), dtype=torch.int64)
    cs = torch.zeros((16, 64), dtype=torch.bfloat16)
    kw = dict(chunk_size=8, max_width=16, rotary_dim=64, is_neox_style=True)
    with pytest.raises(ValueError, match="matching 4-D shapes"):
        f(raw, raw[:1], work, work, plan, cs, **kw)
    with pytest.raises(ValueError, match="contiguous 2-D int64"):
        f(raw, raw, work, work, plan.int(), cs, **kw)
    with pytest.raises(ValueError, match="token capacity"):
        f(raw, raw, work, work, plan, cs, **{**kw, "max_width": 17})
    with pytest.raises(ValueError, match="rotary_dim must be even"):
        f(raw, raw, work, work, plan, cs, **{**kw, "rotary_dim": 3})
    with pytest.raises(ValueError, match="cos/sin cache"):
        f(raw, raw, work, work, plan, cs[:8], **kw)
    with pytest.raises(ValueError, match="same dtype"):
        f(raw, raw, work.half(), work.half(), plan, cs, **kw)
    with pytest.raises(ValueError, match="plan width"):
        f(raw, raw, work, work, plan[:, :6].contiguous(), cs, **kw)
    f(raw, raw, work, work, plan[:0], cs, **kw)  # empty plan: no work, no device needed
    with pytest.raises(ValueError, match="need CUDA tensors"):
        f(raw, raw, work, work, plan, cs, **kw)


def test_selection_validation(dsb):
    s = dsb.selection.select_context_chunks
    with pytest.raises(ValueError, match="one-dimensional"):
        s(torch.zeros((2, 2)), 4, 2, 4)
    with pytest.raises(ValueError, match="non-negative"):
        s(torch.zeros(2), -1, 2, 4)
    with pytest.raises(ValueError, match="chunk-size multiple"):
        s(torch.zeros(2), 4, 2, 3)
    with pytest.raises(ValueError, match="does not match"):
        s(torch.zeros(3), 4, 2, 4)
    with pytest.raises(ValueError, match="need CUDA tensors"):
        s(torch.zeros(2), 4, 2, 4)


def test_gather_and_attention_validation(dsb):
    raw = torch.zeros((4, 16, 2, 64), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="matching 4-D"):
        dsb.kernels.gather_raw_kv_with_local_rope(raw, raw[:2], torch.zeros((1, 2)),
                                                  torch.zeros((1, 4)), torch.zeros((4, 64)), rope_dim=64)
    with pytest.raises(ValueError, match="block table batch size"):
        dsb.kernels.gather_raw_kv_with_local_rope(raw, raw, torch.zeros((2, 2)),
                                                  torch.zeros((1, 4)), torch.zeros((4, 64)), rope_dim=64)
    wk = torch.zeros((2, 2, 32, 64), dtype=torch.bfloat16)
    q = torch.zeros((2, 8, 64), dtype=torch.bfloat16)
    kv = torch.zeros((2, 2, 64), dtype=torch.bfloat16)
    slots = torch.zeros(2, dtype=torch.int32)
    with pytest.raises(ValueError, match="share a dtype"):
        dsb.attention.draft_decode_attention(q.half(), kv, kv, wk, wk, slots, slots, 0.1)
    with pytest.raises(ValueError, match="need CUDA tensors"):
        dsb.attention.draft_decode_attention(q, kv, kv, wk, wk, slots, slots, 0.1)


def test_runtime_budget_and_settings(dsb):
    settings = dsb.runtime.DiffSpecSettings(64, 64, 4, 4, 4, 0.7, False)
    with pytest.raises(ValueError, match="too small"):
        dsb.runtime.DiffSpecDraftCache(settings, max_num_reqs=1, max_model_len=8, num_kv_heads=1,
                                       head_dim=64, target_num_layers=2, dtype=torch.bfloat16,
                                       device=torch.device("cpu"), cos_sin_cache=torch.zeros((8, 64)))
    assert dsb.selection.history_budget(2048, 4, 64) == 1984
