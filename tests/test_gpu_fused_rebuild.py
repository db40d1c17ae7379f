"""Plan + rebuild in one launch (``rebuild_working_cache``) against the
two-launch path (device plan, then rebuild from the plan) and the oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import recipes as R
from oracle import diffspec_oracle as O

pytestmark = pytest.mark.gpu

DTYPES = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


@pytest.fixture(params=["default", "legacy"])
def kernel(request, monkeypatch):
    """The fused kernel, and DSB_REBUILD_LEGACY=1 (the entry point then runs
    plan + row-kernel rebuild)."""
    if request.param == "legacy":
        monkeypatch.setenv("DSB_REBUILD_LEGACY", "1")
    return request.param


def _state(rng, slots, max_len, chunk, budget, hb, sel_stride):
    """Selection state with every kind of slot: no retrieval (-1), empty (0),
    a few chunks, a full budget and more chunks than a plan row carries."""
    n_chunks_max = max_len // chunk
    sel_chunks = np.zeros((slots, sel_stride), np.int32)
    sel_count = np.zeros(slots, np.int32)
    kinds = [-1, 0, 3, hb // chunk, sel_stride]
    for s in range(slots):
        k = kinds[s % len(kinds)]
        if k > 0:
            k = min(k, sel_stride, n_chunks_max)
            sel_chunks[s, :k] = np.sort(rng.choice(n_chunks_max, size=k, replace=False))
        sel_count[s] = k
    return sel_chunks, sel_count


@pytest.mark.parametrize("dtype,hk,d,rot,neox", [
    ("bf16", 4, 128, 128, True),
    ("f16", 2, 64, 64, True),
    ("bf16", 1, 256, 128, True),
    ("bf16", 2, 128, 128, False),
    ("f32", 2, 64, 64, True),
])
def test_fused_equals_plan_then_rebuild(dsb, cuda, kernel, dtype, hk, d, rot, neox):
    rng = np.random.default_rng(hk * 1000 + d)
    slots, max_len, chunk, budget = 12, 1024, 16, 256
    hb = (budget - 5) // chunk * chunk
    width = 5 + budget // chunk
    sel_stride = width - 5 + 3  # wider than a plan row: the capacity flag fires
    sel_chunks, sel_count = _state(rng, slots, max_len, chunk, budget, hb, sel_stride)
    tdt = DTYPES[dtype]
    rk = torch.randn((slots, max_len, hk, d), device=cuda).to(tdt)
    rv = torch.randn_like(rk)
    table = torch.from_numpy(R.round_to(R.cos_sin_table(budget, rot), dtype)).to(cuda).to(
        torch.float32 if dtype == "f32" else tdt)
    rows = 10
    perm = rng.permutation(slots)
    k4 = int(np.flatnonzero(perm == 4)[0])
    perm[2], perm[k4] = perm[k4], perm[2]  # row 2 takes the over-wide selection of slot 4
    row_slots = torch.from_numpy(perm[:rows].astype(np.int32))
    row_slots[7] = -1  # a row without a slot: flagged, rebuilds nothing
    committed = torch.from_numpy(rng.integers(1, max_len, size=rows).astype(np.int32))
    committed[0] = 1  # empty history
    committed[1] = 5  # shorter than a chunk
    args = [t.to(cuda) for t in (row_slots, committed, torch.from_numpy(sel_chunks),
                                 torch.from_numpy(sel_count))]
    base_k = torch.randn((slots, hk, budget, d), device=cuda).to(tdt)
    base_v = torch.randn_like(base_k)

    wk1, wv1 = base_k.clone(), base_v.clone()
    wl1 = torch.full((slots,), -7, dtype=torch.int32, device=cuda)
    plan1, hl1 = dsb.selection.build_history_plan(
        *args, chunk_size=chunk, history_budget=hb, working_budget=budget, working_lens=wl1)
    dsb.compact_kv.rebuild_compact_kv_from_plan(
        rk, rv, wk1, wv1, plan1, table, chunk_size=chunk, max_width=hb, rotary_dim=rot,
        is_neox_style=neox)
    flag1 = dsb._lib.read_and_clear_error_flag(cuda)

    wk2, wv2 = base_k.clone(), base_v.clone()
    wl2 = torch.full((slots,), -7, dtype=torch.int32, device=cuda)
    plan2 = torch.full((rows, width), -9, dtype=torch.int64, device=cuda)
    plan2, hl2 = dsb.compact_kv.rebuild_working_cache(
        rk, rv, wk2, wv2, *args, table, chunk_size=chunk, history_budget=hb, rotary_dim=rot,
        is_neox_style=neox, plan=plan2, working_lens=wl2)
    flag2 = dsb._lib.read_and_clear_error_flag(cuda)

    # the row without a slot (1) and the selection wider than a plan row (16,
    # plus 8 for the prefix positions that row cannot resolve)
    assert flag1 == flag2 and flag1 & 1 and flag1 & 16
    assert torch.equal(plan1, plan2)
    assert torch.equal(hl1, hl2)
    assert torch.equal(wl1, wl2)
    assert torch.equal(wk1.view(torch.uint8), wk2.view(torch.uint8))
    assert torch.equal(wv1.view(torch.uint8), wv2.view(torch.uint8))
    assert int(hl2.max()) > 0


def test_fused_rebuild_vs_oracle(dsb, cuda):
    """Config-1-like rows through the fused launch against the oracle's plan
    and rebuild (bf16, NeoX, reordered slots)."""
    rng = np.random.default_rng(5)
    slots, max_len, hk, d, chunk, budget = 4, 2048, 1, 128, 32, 512
    hb = (budget - 5) // chunk * chunk
    width = 5 + budget // chunk
    raw_k = O.round_to(rng.standard_normal((slots, max_len, hk, d), dtype=np.float32), "bf16")
    raw_v = O.round_to(rng.standard_normal((slots, max_len, hk, d), dtype=np.float32), "bf16")
    table = O.round_to(R.cos_sin_table(budget, d), "bf16")
    sel = [None, [], [3, 9, 40, 61], list(range(0, 60, 4))]
    sel_chunks = np.zeros((slots, width - 5), np.int32)
    sel_count = np.array([-1 if s is None else len(s) for s in sel], np.int32)
    for s, c in enumerate(sel):
        if c:
            sel_chunks[s, : len(c)] = c
    row_slots = np.array([2, 0, 3, 1], np.int32)
    committed = np.array([1990, 700, 2047, 33], np.int32)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    bf = lambda a: dev(a).bfloat16()  # noqa: E731
    wk = torch.zeros((slots, hk, budget, d), device=cuda, dtype=torch.bfloat16)
    wv = torch.zeros_like(wk)
    plan, hl = dsb.compact_kv.rebuild_working_cache(
        bf(raw_k), bf(raw_v), wk, wv, dev(row_slots), dev(committed), dev(sel_chunks),
        dev(sel_count), bf(table), chunk_size=chunk, history_budget=hb, rotary_dim=d,
        is_neox_style=True)
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0
    ref_plan = np.zeros((len(row_slots), width), np.int64)
    for r, s in enumerate(row_slots):
        row = O.history_plan(int(s), sel[s], int(committed[r]) - 1, chunk, hb)
        ref_plan[r, : len(row)] = row
    np.testing.assert_array_equal(plan.cpu().numpy(), ref_plan)
    np.testing.assert_array_equal(hl.cpu().numpy(), ref_plan[:, 1])
    ok_, ov_ = np.zeros((slots, hk, budget, d), np.float32), np.zeros((slots, hk, budget, d), np.float32)
    O.rebuild_compact_kv_from_plan(raw_k, raw_v, ok_, ov_, ref_plan, table, chunk, hb, d, True)
    np.testing.assert_array_equal(wk.float().cpu().numpy(), ok_)
    np.testing.assert_array_equal(wv.float().cpu().numpy(), ov_)
