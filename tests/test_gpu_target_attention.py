"""Target paged decode attention with the softmax LSE exported
(dsb_paged_decode_attention_lse) against the oracle, and the exported LSE
driving the chunk-retrieval scores the way the captured FIA LSE does."""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import diffspec_oracle as O

pytestmark = pytest.mark.gpu

_T = {"bf16": torch.bfloat16, "f16": torch.float16}
_FRAC = {"bf16": 7, "f16": 10}


def _case(rng, dtype, rows, hq, hk, bs, lens, extra_blocks=3):
    d = 128
    cols = max(1, max(-(-n // bs) for n in lens))
    nblocks = rows * cols + extra_blocks
    perm = rng.permutation(nblocks)[: rows * cols].reshape(rows, cols).astype(np.int32)
    kc = O.round_to(rng.standard_normal((nblocks, bs, hk, d), dtype=np.float32), dtype)
    vc = O.round_to(rng.standard_normal((nblocks, bs, hk, d), dtype=np.float32), dtype)
    q = O.round_to(rng.standard_normal((rows, hq, d), dtype=np.float32), dtype)
    return q, kc, vc, perm, np.asarray(lens, dtype=np.int32)


def _run(dsb, cuda, dtype, q, kc, vc, bt, lens, table_rows=None, tps=512):
    dev = lambda a, t=None: torch.from_numpy(np.ascontiguousarray(a)).to(cuda) if t is None \
        else torch.from_numpy(np.ascontiguousarray(a)).to(cuda).to(t)  # noqa: E731
    tr = None if table_rows is None else dev(table_rows)
    out, lse = dsb.kernels.paged_decode_attention_lse(
        dev(q, _T[dtype]), dev(kc, _T[dtype]), dev(vc, _T[dtype]), dev(bt), dev(lens),
        scale=128 ** -0.5, max_seq_len=int(max(lens.max(), 1)), table_rows=tr,
        tokens_per_split=tps)
    torch.cuda.synchronize()
    return out.float().cpu().numpy(), lse.cpu().numpy()


@pytest.mark.parametrize("dtype,hq,hk,lens,tps", [
    ("bf16", 32, 4, [0, 1, 37, 600, 1000], 128),   # config-2 heads, several splits, empty row
    ("f16", 8, 8, [5, 300, 64], 64),               # one query head per kv head
    ("bf16", 16, 1, [513, 2, 700], 512),           # 16 query heads per kv head
    ("bf16", 4, 2, [4096], 256),                   # one long row, 16 splits
    ("bf16", 8, 2, [20000, 16384, 3], 0),          # library default split: 1024 from 16384 on
])
def test_decode_attention_and_lse_match_oracle(dsb, cuda, dtype, hq, hk, lens, tps):
    rng = np.random.default_rng(len(lens) * 97 + hq)
    q, kc, vc, bt, lens = _case(rng, dtype, len(lens), hq, hk, 16, lens)
    out, lse = _run(dsb, cuda, dtype, q, kc, vc, bt, lens, tps=tps)
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0
    ref_out, ref_lse = O.paged_decode_attention_lse(q, kc, vc, bt, lens, 128 ** -0.5, dtype=dtype)
    ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(ref_out), 2.0 ** -14))) - _FRAC[dtype])
    # fp32 accumulation against the oracle's fp64: one ulp of the output, or
    # 1e-5 absolute near zero
    assert (np.abs(out - ref_out) <= np.maximum(ulp, 1e-5)).all()
    empty = lens == 0
    assert np.isneginf(lse[empty]).all() and (out[empty] == 0).all()
    np.testing.assert_allclose(lse[~empty], ref_lse[~empty], rtol=0, atol=2e-5 * max(1, np.abs(ref_lse[~empty]).max()))


def test_table_rows_and_bad_pages(dsb, cuda):
    rng = np.random.default_rng(3)
    q, kc, vc, bt, lens = _case(rng, "bf16", 3, 8, 2, 16, [100, 64, 200])
    rows_map = np.array([2, 2, 0], dtype=np.int32)  # two query rows of one request
    lens = np.array([200, 150, 100], dtype=np.int32)
    out, lse = _run(dsb, cuda, "bf16", q, kc, vc, bt, lens, table_rows=rows_map, tps=64)
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0
    ref_out, ref_lse = O.paged_decode_attention_lse(q, kc, vc, bt, lens, 128 ** -0.5,
                                                    table_rows=rows_map)
    np.testing.assert_allclose(out, ref_out, rtol=1e-2, atol=1e-2)
    np.testing.assert_allclose(lse, ref_lse, atol=1e-4)
    bad = bt.copy()
    bad[2, 1] = 10 ** 6  # a page entry past the cache: flagged, its tokens skipped
    _run(dsb, cuda, "bf16", q, kc, vc, bad, lens, table_rows=rows_map, tps=64)
    assert dsb._lib.read_and_clear_error_flag(cuda) & 4  # DSB_FLAG_BLOCK


def test_exported_lse_drives_retrieval_scores(dsb, cuda):
    """Chunk scores with the exported LSE equal the ones whose LSE the scores
    pass computes itself (softmax_lse=None), as the captured FIA LSE would."""
    rng = np.random.default_rng(11)
    lens_l = [2000, 1500, 64, 777]
    q, kc, vc, bt, lens = _case(rng, "bf16", 4, 32, 4, 16, lens_l)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    qt, kt, vt = dev(q).bfloat16(), dev(kc).bfloat16(), dev(vc).bfloat16()
    _, lse = dsb.kernels.paged_decode_attention_lse(qt, kt, vt, dev(bt), dev(lens),
                                                    scale=128 ** -0.5, max_seq_len=2000)
    kw = dict(chunk_size=64, max_seq_len=2000, scale=128 ** -0.5)
    with_lse = dsb.kernels.paged_chunk_attention_scores(qt, kt, lse, dev(bt), dev(lens), **kw)
    own = dsb.kernels.paged_chunk_attention_scores(qt, kt, None, dev(bt), dev(lens), **kw)
    torch.cuda.synchronize()
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0
    np.testing.assert_allclose(with_lse.cpu().numpy(), own.cpu().numpy(), rtol=1e-3, atol=1e-7)


def test_runtime_runs_target_attention_and_captures_its_lse(dsb, cuda):
    """DiffSpecDraftCache.run_target_attention: causal verify spans of three
    rows per request, the output against the oracle, the captured LSE used by
    the next retrieval."""
    rng = np.random.default_rng(17)
    seq_lens = [300, 150]
    q, kc, vc, bt, _ = _case(rng, "bf16", 6, 8, 1, 16, seq_lens)
    bt = bt[:2]
    settings = dsb.runtime.DiffSpecSettings(16, 128, 1, 4, 3, 0.7, False)
    cache = dsb.runtime.DiffSpecDraftCache(
        settings, max_num_reqs=2, max_model_len=512, num_kv_heads=1, head_dim=128,
        target_num_layers=2, dtype=torch.bfloat16, device=cuda,
        cos_sin_cache=torch.zeros((128, 128), device=cuda).bfloat16())
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    meta = SimpleNamespace(actual_seq_lengths_q=[3, 6], seq_lens_list=seq_lens,
                           block_tables=dev(bt), num_prefills=0)
    cache.begin_target_forward(["a", "b"])
    qt = dev(q).bfloat16()
    out = cache.run_target_attention(qt, dev(kc).bfloat16(), dev(vc).bfloat16(), meta, 128 ** -0.5)
    torch.cuda.synchronize()
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0
    visible = np.array([298, 299, 300, 148, 149, 150])
    ref_out, ref_lse = O.paged_decode_attention_lse(q, kc, vc, bt, visible, 128 ** -0.5,
                                                    table_rows=np.array([0, 0, 0, 1, 1, 1]))
    np.testing.assert_allclose(out.float().cpu().numpy(), ref_out, rtol=1e-2, atol=1e-2)
    np.testing.assert_allclose(cache._target["lse"].cpu().numpy(), ref_lse, atol=1e-4)
    cache.accept_target_queries(torch.tensor([2, 3], device=cuda), is_prefill=False)
    assert cache.retrieval_status()["retrieval_count"] == 1
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0


def test_rows_beyond_max_seq_len_are_flagged_and_cut(dsb, cuda):
    """A max_seq_len below a row's length cannot cover it with splits: the
    row is cut at the splits' reach (64 tokens here) and DSB_FLAG_POSITION
    is raised instead of silently dropping the tail."""
    rng = np.random.default_rng(23)
    q, kc, vc, bt, _ = _case(rng, "bf16", 1, 8, 2, 16, [100])
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    out, lse = dsb.kernels.paged_decode_attention_lse(
        dev(q).bfloat16(), dev(kc).bfloat16(), dev(vc).bfloat16(), dev(bt),
        dev(np.array([100], np.int32)), scale=128 ** -0.5, max_seq_len=50, tokens_per_split=16)
    torch.cuda.synchronize()
    assert dsb._lib.read_and_clear_error_flag(cuda) == 2  # DSB_FLAG_POSITION
    ref_out, ref_lse = O.paged_decode_attention_lse(q, kc, vc, bt, np.array([64]), 128 ** -0.5)
    np.testing.assert_allclose(out.float().cpu().numpy(), ref_out, rtol=1e-2, atol=1e-2)
    np.testing.assert_allclose(lse.cpu().numpy(), ref_lse, atol=1e-4)
