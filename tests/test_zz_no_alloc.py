"""The allocation-free draft attention entry point, called through the C ABI.

dsb_draft_decode_attention_static serves callers that cannot allocate device
memory when the draft step runs (an engine that pre-reserves its memory, a
step being recorded into a CUDA graph, a latency budget that cannot absorb a
synchronising cudaMalloc).  It keeps its split scratch in library-owned
static device arrays; this test checks that two consecutive calls give the
output of the allocating entry point within the path's bf16 tolerance.
The file is named to be collected last.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import recipes as R
from conftest import close_bf16

pytestmark = pytest.mark.gpu


def _static_call(dsb, q, k, v, wk, wv, slots, pos, offset, out, scale):
    lib = dsb._lib.load()
    rows = slots.shape[0]
    s, hk, w, d = wk.shape
    flag = dsb._lib.error_flag(q.device)
    st = lib.dsb_draft_decode_attention_static(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), wk.data_ptr(), wv.data_ptr(), slots.data_ptr(),
        pos.data_ptr(), offset, rows, out.shape[0], s, q.shape[1], hk, d, w, ctypes.c_float(scale),
        dsb._lib.DSB_BF16, out.data_ptr(), 0, flag.data_ptr(),
        ctypes.c_void_p(torch.cuda.current_stream(q.device).cuda_stream))
    dsb._lib.check(st, "dsb_draft_decode_attention_static")


def test_static_scratch_attention_matches_allocating_entry_point(dsb, cuda):
    g = R.rng(4242)
    slots_n, hk, hq, d, w = 18, 4, 32, 128, 2048
    bf = lambda a: torch.from_numpy(a).to(cuda).bfloat16()  # noqa: E731
    wk0 = bf(R.normal(g, (slots_n, hk, w, d), "bf16"))
    wv0 = bf(R.normal(g, (slots_n, hk, w, d), "bf16"))
    slots = torch.tensor([17, 3, 0, 9, 12, 1, 5, 16, 2, 8, 11, 4, 15, 7, 10, 6],
                         dtype=torch.int32, device=cuda)
    pos = torch.tensor([1984 - 3 * i for i in range(16)], dtype=torch.int32, device=cuda)
    scale = d ** -0.5
    wk_a, wv_a = wk0.clone(), wv0.clone()
    wk_b, wv_b = wk0.clone(), wv0.clone()
    for step in range(2):  # two calls in a row, as consecutive draft steps
        q = bf(R.normal(g, (18, hq, d), "bf16"))
        k = bf(R.normal(g, (16, hk, d), "bf16"))
        v = bf(R.normal(g, (16, hk, d), "bf16"))
        ref = torch.full((18, hq, d), float("nan"), device=cuda).bfloat16()
        dsb.attention.draft_decode_attention(q, k, v, wk_a, wv_a, slots, pos, scale, ref, rows=16,
                                             position_offset=step)
        out = torch.full((18, hq, d), float("nan"), device=cuda).bfloat16()
        _static_call(dsb, q, k, v, wk_b, wv_b, slots, pos, step, out, scale)
        torch.cuda.synchronize()
        close_bf16(out.float().cpu().numpy(), ref.float().cpu().numpy())
        np.testing.assert_allclose(out.float().cpu().numpy(), ref.float().cpu().numpy(),
                                   rtol=0.03, atol=0.02)
        assert torch.equal(wk_a, wk_b) and torch.equal(wv_a, wv_b)
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0


def test_static_scratch_rejects_oversized_calls(dsb, cuda):
    lib = dsb._lib.load()
    x = torch.zeros(16, device=cuda)
    p = x.data_ptr()
    # 2048 rows x 4 kv heads = 8192 tickets > 4096
    st = lib.dsb_draft_decode_attention_static(p, p, p, p, p, p, p, 0, 2048, 2048, 2048, 32, 4, 128,
                                               2048, ctypes.c_float(0.1), 0, p, 0, None, None)
    assert st == dsb._lib.DSB_ERR_INVALID
    assert b"4096" in lib.dsb_last_error()
    # 512 rows x 4 kv heads x 64 splits of partials exceeds the 4 MiB scratch
    st = lib.dsb_draft_decode_attention_static(p, p, p, p, p, p, p, 0, 512, 512, 512, 32, 4, 128,
                                               2048, ctypes.c_float(0.1), 0, p, 64, None, None)
    assert st == dsb._lib.DSB_ERR_INVALID
    assert b"static scratch" in lib.dsb_last_error()
