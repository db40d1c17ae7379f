"""Fused gather + local-RoPE kernels (rows A6, A7) against reference and oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import recipes as R
from conftest import close_bf16, from_bits, golden
from oracle import diffspec_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True, params=["bulk", "legacy"])
def kernel(request, monkeypatch):
    """Run every case on the bulk-copy kernel (default) and on the cp.async
    row kernel the library falls back to."""
    if request.param == "legacy":
        monkeypatch.setenv("DSB_REBUILD_LEGACY", "1")
    return request.param


def bf16(a, device):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device).bfloat16()


def f32(t):
    return t.float().cpu().numpy()


@pytest.fixture(scope="module")
def rebuild():
    return golden("rebuild")


@pytest.mark.parametrize("k", range(len(R.REBUILD_CASES) * len(R.REBUILD_ENDS)))
def test_rebuild_matches_reference_and_oracle(dsb, cuda, rebuild, k):
    p = f"case{k}_"
    ci, end, max_width = (int(v) for v in rebuild[p + "meta"])
    inp = R.rebuild_inputs(ci)
    plan = rebuild[p + "plan"]
    rk, rv = bf16(inp["raw_key"], cuda), bf16(inp["raw_value"], cuda)
    shape = (R.REBUILD_SLOTS, inp["heads"], R.REBUILD_BUDGET, inp["dim"])
    wk = torch.full(shape, float("nan"), device=cuda).bfloat16()
    wv = wk.clone()
    dsb.compact_kv.rebuild_compact_kv_from_plan(
        rk, rv, wk, wv, torch.from_numpy(plan).to(cuda), bf16(inp["cos_sin"], cuda),
        chunk_size=R.REBUILD_CHUNK, max_width=max_width, rotary_dim=inp["rot"],
        is_neox_style=inp["neox"])
    torch.cuda.synchronize()
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0
    ok, ov = (np.full(shape, np.nan, np.float32) for _ in range(2))
    O.rebuild_compact_kv_from_plan(inp["raw_key"], inp["raw_value"], ok, ov, plan, inp["cos_sin"],
                                   R.REBUILD_CHUNK, max_width, inp["rot"], inp["neox"], "bf16")
    gk, gv = f32(wk), f32(wv)
    np.testing.assert_array_equal(gk, ok)  # bit-exact vs the oracle (NaN where untouched)
    np.testing.assert_array_equal(gv, ov)
    for r, slot in enumerate(inp["slots"]):
        h = int(plan[r][1])
        ref = from_bits(rebuild, p + f"row{r}_ref_triton_wk")
        ulp = np.abs(gk[slot, :, :h].view(np.int32).astype(np.int64) - ref.view(np.int32).astype(np.int64))
        assert ulp.max(initial=0) <= 1 << 16  # interpreter truncates, hardware rounds
        if end >= 62:
            close_bf16(gk[slot, :, :h], from_bits(rebuild, p + f"row{r}_ref_cpu_wk"))
    assert torch.equal(rk, bf16(inp["raw_key"], cuda)) and torch.equal(rv, bf16(inp["raw_value"], cuda))


def test_config2_rebuild_rows_vs_oracle(dsb, cuda):
    """Config-2 geometry (max_model_len 40960, 4 kv heads, D 128, W 2048,
    C 64, history budget 1984) for 4 slots in reordered order."""
    slots_n, length, hk, d, w, c, hb = 4, 40960, 4, 128, 2048, 64, 1984
    g = R.rng(202)
    raw_k = R.normal(g, (slots_n, length, hk, d), "bf16")
    raw_v = R.normal(g, (slots_n, length, hk, d), "bf16")
    table = R.round_to(R.cos_sin_table(w, d), "bf16")
    rows = []
    for slot in (3, 1, 0, 2):
        n = 600 + 10 * slot
        chunks = sorted(g.choice(n - 1, hb // c - 1, replace=False).tolist()) + [n - 1]
        he = n * c - int(g.integers(0, 2 * c))
        rows.append(O.history_plan(slot, chunks, he, c, hb))
    width = 5 + w // c
    plan = np.zeros((4, width), np.int64)
    for r, pl in enumerate(rows):
        plan[r, : len(pl)] = pl
    wk = torch.zeros((slots_n, hk, w, d), device=cuda).bfloat16()
    wv = torch.zeros_like(wk)
    dsb.compact_kv.rebuild_compact_kv_from_plan(
        bf16(raw_k, cuda), bf16(raw_v, cuda), wk, wv, torch.from_numpy(plan).to(cuda),
        bf16(table, cuda), chunk_size=c, max_width=hb, rotary_dim=d, is_neox_style=True)
    ok, ov = np.zeros((slots_n, hk, w, d), np.float32), np.zeros((slots_n, hk, w, d), np.float32)
    O.rebuild_compact_kv_from_plan(raw_k, raw_v, ok, ov, plan, table, c, hb, d, True, "bf16")
    np.testing.assert_array_equal(f32(wk), ok)
    np.testing.assert_array_equal(f32(wv), ov)
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("hk,d,rot,neox", [(8, 128, 128, True), (1, 64, 64, True), (2, 256, 256, True),
                                           (4, 128, 64, True), (4, 64, 64, False)])
def test_rebuild_geometries_vs_oracle(dsb, cuda, dtype, hk, d, rot, neox):
    """Chunk 64 plans with a dropped prefix head, partial last chunks and a
    rolling tail, over head counts that change the positions per CTA."""
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float16
    slots_n, length, w, c, hb = 3, 4096, 512, 64, 448
    g = R.rng(hk * 1000 + d + rot + int(neox))
    raw_k = R.normal(g, (slots_n, length, hk, d), dtype)
    raw_v = R.normal(g, (slots_n, length, hk, d), dtype)
    table = R.round_to(R.cos_sin_table(w, rot), dtype)
    rows = []
    for slot, n_sel, he in ((2, 7, 3001), (0, 3, 1000), (1, 0, 200)):
        n = (he + c) // c
        chunks = sorted(g.choice(n - 1, n_sel, replace=False).tolist()) + [n - 1] if n_sel else []
        rows.append(O.history_plan(slot, chunks, he, c, hb))
    plan = np.zeros((3, 5 + w // c), np.int64)
    for r, pl in enumerate(rows):
        plan[r, : len(pl)] = pl
    wk = torch.full((slots_n, hk, w, d), float("nan"), device=cuda).to(tdt)
    wv = wk.clone()
    dsb.compact_kv.rebuild_compact_kv_from_plan(
        torch.from_numpy(raw_k).to(cuda, tdt), torch.from_numpy(raw_v).to(cuda, tdt), wk, wv,
        torch.from_numpy(plan).to(cuda), torch.from_numpy(table).to(cuda, tdt), chunk_size=c,
        max_width=hb, rotary_dim=rot, is_neox_style=neox)
    ok, ov = (np.full((slots_n, hk, w, d), np.nan, np.float32) for _ in range(2))
    O.rebuild_compact_kv_from_plan(raw_k, raw_v, ok, ov, plan, table, c, hb, rot, neox, dtype)
    np.testing.assert_array_equal(f32(wk), ok)  # NaN where the plan leaves rows untouched
    np.testing.assert_array_equal(f32(wv), ov)
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0


def test_bad_plan_rows_are_flagged_and_skipped(dsb, cuda):
    rk = torch.randn((2, 64, 1, 64), device=cuda).bfloat16()
    rv = torch.randn_like(rk)
    wk = torch.zeros((2, 1, 32, 64), device=cuda).bfloat16()
    wv = torch.zeros_like(wk)
    cs = torch.ones((32, 64), device=cuda).bfloat16()
    plan = torch.zeros((2, 5 + 32 // 8), dtype=torch.int64)
    plan[0, :5] = torch.tensor([0, 10, 60, 0, 0])  # tail runs past max_model_len
    plan[1, :5] = torch.tensor([1, 8, 0, 8, 0])
    plan[1, 5] = 50  # chunk 50 * 8 = 400 >= 64
    dsb.compact_kv.rebuild_compact_kv_from_plan(rk, rv, wk, wv, plan.to(cuda), cs, chunk_size=8,
                                                max_width=10, rotary_dim=64, is_neox_style=True)
    torch.cuda.synchronize()
    flag = dsb._lib.read_and_clear_error_flag(cuda)
    assert flag & 2
    assert torch.equal(wv[1], torch.zeros_like(wv[1]))
    assert torch.equal(wv[0, :, :4], rv[0, 60:64].transpose(0, 1))


@pytest.mark.parametrize("i", range(len(R.GATHER_CASES)))
def test_gather_matches_reference_and_oracle(dsb, cuda, i):
    d = golden("gather")
    inp = R.gather_inputs(i)
    k, v = dsb.kernels.gather_raw_kv_with_local_rope(
        bf16(inp["raw_key"], cuda), bf16(inp["raw_value"], cuda),
        torch.from_numpy(inp["block_table"]).to(cuda), torch.from_numpy(inp["selected"]).to(cuda),
        bf16(inp["cos_sin"], cuda), rope_dim=inp["rot"], is_neox_style=inp["neox"])
    torch.cuda.synchronize()
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0
    np.testing.assert_array_equal(f32(v), from_bits(d, f"case{i}_ref_value"))
    np.testing.assert_array_equal(f32(k), from_bits(d, f"case{i}_ref_key"))
    ok, ov = O.gather_raw_kv_with_local_rope(inp["raw_key"], inp["raw_value"], inp["block_table"],
                                             inp["selected"], inp["cos_sin"], inp["rot"], inp["neox"])
    np.testing.assert_array_equal(f32(k), ok)


def test_gather_fp32_table_and_partial_rotary(dsb, cuda):
    g = R.rng(5)
    raw_k = R.normal(g, (6, 16, 2, 128), "bf16")
    raw_v = R.normal(g, (6, 16, 2, 128), "bf16")
    table = np.array([[5, 2, 0], [1, 3, 4]], np.int32)
    sel = g.integers(-1, 48, size=(2, 40)).astype(np.int64)
    cs = R.cos_sin_table(64, 96)
    k, v = dsb.kernels.gather_raw_kv_with_local_rope(
        bf16(raw_k, cuda), bf16(raw_v, cuda), torch.from_numpy(table).to(cuda),
        torch.from_numpy(sel).to(cuda), torch.from_numpy(cs).to(cuda), rope_dim=96,
        is_neox_style=False)
    ok, ov = O.gather_raw_kv_with_local_rope(raw_k, raw_v, table, sel, cs, 96, False)
    np.testing.assert_array_equal(f32(k), ok)
    np.testing.assert_array_equal(f32(v), ov)
