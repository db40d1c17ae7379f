"""Draft decode attention (row A8) against the reference CPU loop and the oracle.

Tolerance (bf16 I/O, fp32 softmax): the path's bound of max abs error
<= 2e-2 * max(1, max|ref|) and mean abs error <= 2e-3 * mean|ref|, plus the
reference device test's own rtol=0.03 / atol=0.02
(tests/test_linear_attention_batch_npu.py:136)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import recipes as R
from conftest import close_bf16, golden
from oracle import diffspec_oracle as O

pytestmark = pytest.mark.gpu


def bf16(a, device):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device).bfloat16()


KERNELS = ["tma", "tma-ticket", "legacy"]


def use_kernel(kernel, monkeypatch):
    """tma: TMA-fed kernel on mma.sync (the default); tma-ticket: splits
    merged through global partials and an atomic ticket instead of inside a
    thread-block cluster; legacy: the register-fed kernel the library falls
    back to."""
    if kernel == "legacy":
        monkeypatch.setenv("DSB_ATTENTION_LEGACY", "1")
    if kernel.endswith("-ticket"):
        monkeypatch.setenv("DSB_ATTENTION_TICKET_MERGE", "1")


@pytest.mark.parametrize("i", range(len(R.attention_cases())))
@pytest.mark.parametrize("splits", [None, 1, 2, 3])
@pytest.mark.parametrize("kernel", KERNELS)
def test_attention_matches_reference(dsb, cuda, i, splits, kernel, monkeypatch):
    use_kernel(kernel, monkeypatch)
    d = golden("attention")
    inp = R.attention_inputs(i)
    n = len(inp["slots"])
    wk, wv = bf16(inp["working_key"], cuda), bf16(inp["working_value"], cuda)
    slots = torch.tensor(inp["slots"], dtype=torch.int32, device=cuda)
    base = torch.tensor(inp["positions"], dtype=torch.int32, device=cuda)
    for step, st in enumerate(inp["steps"]):
        out = torch.full((R.ATTN_ROWS, inp["qheads"], inp["dim"]), float("nan"), device=cuda).bfloat16()
        dsb.attention.draft_decode_attention(
            bf16(st["query"], cuda), bf16(st["key"], cuda), bf16(st["value"], cuda), wk, wv,
            slots, base, inp["dim"] ** -0.5, out, rows=n, position_offset=step, num_splits=splits)
        got = out.float().cpu().numpy()
        ref = d[f"case{i}_step{step}_ref_out"]
        close_bf16(got, ref)
        np.testing.assert_allclose(got, ref, rtol=0.03, atol=0.02)
        assert not got[n:].any()  # graph-padding rows are zero
        for r, slot in enumerate(inp["slots"]):
            pos = inp["positions"][r] + step
            assert torch.equal(wk[slot, :, pos], bf16(st["key"][r], cuda))
            assert torch.equal(wv[slot, :, pos], bf16(st["value"][r], cuda))
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("hq,hk,d", [(32, 4, 128), (64, 8, 128), (16, 1, 128), (8, 2, 64),
                                     (16, 2, 256), (32, 2, 128)])
@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("splits", [None, 2, 5, 8, 12])
def test_long_history_split_kv_vs_oracle(dsb, cuda, dtype, hq, hk, d, kernel, splits, monkeypatch):
    """Config-2 lengths (history 1984 + draft step) with reordered slots; rows
    whose history ends before the last splits leave those splits empty."""
    use_kernel(kernel, monkeypatch)
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float16
    g = R.rng(hq * 131 + hk + d)
    slots_n, w = 6, 2048
    wk = R.normal(g, (slots_n, hk, w, d), dtype)
    wv = R.normal(g, (slots_n, hk, w, d), dtype)
    slots = [4, 0, 5, 2]
    positions = [1984, 1987, 700, 0]
    q = R.normal(g, (4, hq, d), dtype) * 2.0
    k = R.normal(g, (4, hk, d), dtype)
    v = R.normal(g, (4, hk, d), dtype)
    twk = torch.from_numpy(wk).to(cuda, tdt)
    twv = torch.from_numpy(wv).to(cuda, tdt)
    out = dsb.attention.draft_decode_attention(
        torch.from_numpy(q).to(cuda, tdt), torch.from_numpy(k).to(cuda, tdt),
        torch.from_numpy(v).to(cuda, tdt), twk, twv,
        torch.tensor(slots, dtype=torch.int32, device=cuda),
        torch.tensor(positions, dtype=torch.int32, device=cuda), d ** -0.5, num_splits=splits)
    ref = O.draft_decode_attention(q, k, v, wk, wv, slots, positions, d ** -0.5, dtype=None)
    close_bf16(out.float().cpu().numpy(), ref)
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0


def test_repeated_calls_leave_merge_tickets_clean(dsb, cuda):
    """The split-merge tickets return to zero after every call, so the same
    workspace gives identical results call after call."""
    g = R.rng(9)
    wk = bf16(R.normal(g, (16, 4, 2048, 128), "bf16"), cuda)
    wv = bf16(R.normal(g, (16, 4, 2048, 128), "bf16"), cuda)
    q = bf16(R.normal(g, (16, 32, 128), "bf16"), cuda)
    k = bf16(R.normal(g, (16, 4, 128), "bf16"), cuda)
    v = bf16(R.normal(g, (16, 4, 128), "bf16"), cuda)
    slots = torch.arange(16, dtype=torch.int32, device=cuda)
    pos = torch.full((16,), 1985, dtype=torch.int32, device=cuda)
    ws = dsb.attention.AttentionWorkspace(cuda)
    outs = [dsb.attention.draft_decode_attention(q, k, v, wk, wv, slots, pos, 0.088, workspace=ws)
            for _ in range(3)]
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])
    assert not ws.counters.any()


def test_bad_slot_or_position_is_flagged_with_zero_output(dsb, cuda):
    wk = torch.randn((2, 1, 64, 64), device=cuda).bfloat16()
    wv = torch.randn_like(wk)
    q = torch.randn((2, 8, 64), device=cuda).bfloat16()
    k = torch.randn((2, 1, 64), device=cuda).bfloat16()
    out = dsb.attention.draft_decode_attention(
        q, k, k, wk, wv, torch.tensor([5, 0], dtype=torch.int32, device=cuda),
        torch.tensor([3, 64], dtype=torch.int32, device=cuda), 0.125)
    torch.cuda.synchronize()
    flag = dsb._lib.read_and_clear_error_flag(cuda)
    assert flag & 1 and flag & 2
    assert not out.float().any()
