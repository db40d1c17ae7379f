"""DraftPeriodGraph: a retrieval period captured as one CUDA graph, host
copies included, against the same period run through the cache's methods
eagerly: selections, working caches and every draft step's output must be
the same bits, over two periods whose lengths and inputs differ."""

from __future__ import annotations

import pytest
import torch

import recipes as R

pytestmark = pytest.mark.gpu

N, HQ, HK, D, BS, C, BUDGET, DEPTH, INTERVAL, CTX = 4, 16, 2, 128, 16, 32, 512, 4, 2, 2048


def _cache(dsb, cuda):
    settings = dsb.runtime.DiffSpecSettings(C, BUDGET, INTERVAL, 4, DEPTH, 0.7, False)
    table = torch.from_numpy(R.round_to(R.cos_sin_table(BUDGET, D), "bf16")).bfloat16()
    return dsb.runtime.DiffSpecDraftCache(
        settings, max_num_reqs=N + 2, max_model_len=CTX + 64, num_kv_heads=HK, head_dim=D,
        target_num_layers=2, dtype=torch.bfloat16, device=cuda, cos_sin_cache=table,
        rotary_dim=D, is_neox_style=True, recent_window=2 * C)


def _period_inputs(g, seed):
    """Verify-pass blocks and draft-step q/k/v of one period (host tensors)."""
    gen = torch.Generator().manual_seed(seed)
    bf = torch.bfloat16
    verify, steps = [], []
    for c in range(INTERVAL):
        seq = torch.randint(CTX // 2, CTX + 1, (N,), generator=gen).to(torch.int32)
        verify.append(dict(
            query=torch.randn((5 * N, HQ, D), generator=gen).to(bf),
            lse=torch.rand((5 * N, HQ), generator=gen) + 8.0,
            counts=torch.randint(0, 5, (N,), generator=gen).to(torch.int64),
            query_ends=(torch.arange(1, N + 1) * 5).to(torch.int32),
            seq_lens=seq,
            committed=(seq - torch.randint(0, 4, (N,), generator=gen)).to(torch.int32)))
        steps.append([dict(q=torch.randn((N, HQ, D), generator=gen).to(bf),
                           k=torch.randn((N, HK, D), generator=gen).to(bf),
                           v=torch.randn((N, HK, D), generator=gen).to(bf))
                      for _ in range(DEPTH)])
    return verify, steps


def test_period_graph_matches_eager_methods(dsb, cuda):
    gen = torch.Generator(device=cuda).manual_seed(5)
    pages = CTX // BS
    key_cache = torch.randn((N * pages, BS, HK, D), generator=gen, device=cuda).bfloat16()
    block_tables = torch.randperm(N * pages, generator=gen, device=cuda).to(torch.int32).view(N, pages)
    ids = [f"r{i}" for i in range(N)]
    caches = [_cache(dsb, cuda) for _ in range(2)]
    raw_k = torch.randn(caches[0].raw_key.shape, generator=gen, device=cuda).bfloat16()
    raw_v = torch.randn(caches[0].raw_key.shape, generator=gen, device=cuda).bfloat16()
    for cache in caches:
        cache.raw_key.copy_(raw_k)
        cache.raw_value.copy_(raw_v)
        cache.working_key.zero_()  # compared whole below, rows no period writes included
        cache.working_value.zero_()
        cache.set_active_requests(["pad"] + ids)  # slots 1..N: the slot vector is not the identity
        cache.set_active_requests(ids)
    eager, graphed = caches
    g = dsb.runtime.DraftPeriodGraph(graphed, ids, key_cache=key_cache, block_tables=block_tables,
                                     query_rows_per_request=5, num_query_heads=HQ,
                                     max_seq_len=CTX, scale=D ** -0.5)
    assert g.h2d_bytes > 0 and g.d2h_bytes == INTERVAL * DEPTH * N * HQ * D * 2
    out = torch.empty((N, HQ, D), dtype=torch.bfloat16, device=cuda)
    for period, seed in enumerate((11, 12)):
        verify, steps = _period_inputs(g, seed)
        for c in range(INTERVAL):
            for name, t in verify[c].items():
                g.inputs["verify"][c][name].copy_(t)
            for j in range(DEPTH):
                for name, t in steps[c][j].items():
                    g.inputs["step"][c][j][name].copy_(t)
        g.replay()
        g.done.synchronize()
        # the same period through the cache's methods
        v0 = verify[0]
        eager.retrieve(v0["query"].to(cuda), v0["lse"].to(cuda), key_cache, block_tables,
                       v0["query_ends"].tolist(), v0["seq_lens"].tolist(), v0["counts"].to(cuda),
                       D ** -0.5)
        for c in range(INTERVAL):
            eager.begin_cycle(ids)
            eager.rebuild(verify[c]["committed"].tolist())
            for j in range(DEPTH):
                st = {k: t.to(cuda) for k, t in steps[c][j].items()}
                eager.forward_attention(st["q"], st["k"], st["v"], D ** -0.5, out)
                assert torch.equal(g.outputs[c, j], out.cpu()), (period, c, j)
            eager.end_cycle()
        torch.cuda.synchronize()
        assert torch.equal(graphed.sel_count, eager.sel_count)
        assert torch.equal(graphed.sel_chunks, eager.sel_chunks)
        assert torch.equal(graphed.working_key, eager.working_key)
        assert torch.equal(graphed.working_value, eager.working_value)
        assert torch.equal(graphed._history_lens, eager._history_lens)
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0
