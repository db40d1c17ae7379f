"""Draft-layer K/V projection with the raw-cache write in its epilogue
(dsb_kv_projection_write_raw) against the oracle's projection + _write_raw."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import diffspec_oracle as O

pytestmark = pytest.mark.gpu

_T = {"bf16": torch.bfloat16, "f16": torch.float16}


@pytest.fixture(autouse=True, params=["ranks16", "ranks8"])
def cluster_size(request, monkeypatch):
    """Every case with the default 16-CTA split-K clusters and with the 8-CTA
    ones (DSB_KV_PROJECTION_RANKS8=1)."""
    if request.param == "ranks8":
        monkeypatch.setenv("DSB_KV_PROJECTION_RANKS8", "1")
    return request.param
_FRAC = {"bf16": 7, "f16": 10}  # fraction bits of the stored type


def within_one_ulp(got, ref_f32, dtype):
    """|got - ref| <= one unit in the last place of the stored type at |ref|
    (the fp32 sums differ only in order from the oracle's)."""
    mag = np.maximum(np.abs(ref_f32), 2.0 ** -14)
    ulp = np.exp2(np.floor(np.log2(mag)) - _FRAC[dtype])
    return np.abs(got - ref_f32) <= ulp


@pytest.mark.parametrize("dtype,tokens,hidden,hk,d", [
    ("bf16", 16, 4096, 4, 128),   # config-5 decode step: Eagle3 qkv input 4096, 4 kv heads
    ("bf16", 37, 512, 2, 64),     # three token tiles, ragged last one
    ("f16", 5, 1024, 1, 128),     # fewer tokens than a tile, ranks with one k-block each
    ("bf16", 20, 256, 4, 128),    # fewer k-blocks than cluster ranks
])
def test_projection_and_raw_write_match_oracle(dsb, cuda, dtype, tokens, hidden, hk, d):
    rng = np.random.default_rng(tokens * 31 + hidden)
    slots_n, max_len = 24, 300
    h = O.round_to(rng.standard_normal((tokens, hidden), dtype=np.float32), dtype)
    w = O.round_to(rng.standard_normal((2 * hk * d, hidden), dtype=np.float32) / np.sqrt(hidden), dtype)
    slots = rng.permutation(slots_n)[:tokens].astype(np.int32) if tokens <= slots_n else \
        (np.arange(tokens) % slots_n).astype(np.int32)
    slots[1] = -1  # a padding row: no cache row
    positions = rng.integers(0, max_len, size=tokens).astype(np.int64)
    if tokens > slots_n:  # distinct (slot, position) cells
        positions = (np.arange(tokens) // slots_n * 97 + 3).astype(np.int64)
    raw_k0 = O.round_to(rng.standard_normal((slots_n, max_len, hk, d), dtype=np.float32), dtype)
    raw_v0 = O.round_to(rng.standard_normal((slots_n, max_len, hk, d), dtype=np.float32), dtype)
    tdt = _T[dtype]
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    rk, rv = dev(raw_k0).to(tdt), dev(raw_v0).to(tdt)
    out = dsb.kernels.kv_projection_write_raw(dev(h).to(tdt), dev(w).to(tdt), dev(slots),
                                              dev(positions), rk, rv)
    torch.cuda.synchronize()
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0
    ok_, ov_ = raw_k0.copy(), raw_v0.copy()
    ref = O.kv_projection_write_raw(h, w, slots, positions, ok_, ov_, dtype)
    ref_f32 = h.astype(np.float64) @ w.astype(np.float64).T
    got = out.float().cpu().numpy()
    assert within_one_ulp(got, ref_f32, dtype).all()
    assert (got == ref).mean() > 0.99  # nearly all round the same way as the oracle
    # the cache rows hold exactly the returned rows; every other row is untouched
    half = hk * d
    gk, gv = rk.float().cpu().numpy(), rv.float().cpu().numpy()
    exp_k, exp_v = raw_k0.copy(), raw_v0.copy()
    for t in range(tokens):
        if slots[t] >= 0:
            exp_k[slots[t], positions[t]] = got[t, :half].reshape(hk, d)
            exp_v[slots[t], positions[t]] = got[t, half:].reshape(hk, d)
    np.testing.assert_array_equal(gk, exp_k)
    np.testing.assert_array_equal(gv, exp_v)


def test_bad_cache_cells_are_flagged_and_skipped(dsb, cuda):
    tokens, hidden, hk, d, slots_n, max_len = 4, 256, 1, 128, 3, 50
    g = torch.Generator(device="cpu").manual_seed(7)
    h = torch.randn((tokens, hidden), generator=g).bfloat16().to(cuda)
    w = torch.randn((2 * hk * d, hidden), generator=g).bfloat16().to(cuda)
    rk = torch.zeros((slots_n, max_len, hk, d), device=cuda).bfloat16()
    rv = torch.zeros_like(rk)
    slots = torch.tensor([0, 5, 1, 2], dtype=torch.int32, device=cuda)       # 5: no such slot
    pos = torch.tensor([3, 4, max_len, 9], dtype=torch.int64, device=cuda)   # max_len: out of range
    out = dsb.kernels.kv_projection_write_raw(h, w, slots, pos, rk, rv)
    flag = dsb._lib.read_and_clear_error_flag(cuda)
    assert flag & 1 and flag & 2  # slot and position bits
    assert torch.equal(rk[0, 3].reshape(-1), out[0, :d]) and torch.equal(rk[2, 9].reshape(-1), out[3, :d])
    assert int((rk != 0).sum()) == 2 * d and int((rv != 0).sum()) == 2 * d


def test_runtime_projection_writes_the_draft_cache(dsb, cuda):
    """DiffSpecDraftCache.project_and_write_raw fills its own raw caches with
    the rows the kernel returns."""
    settings = dsb.runtime.DiffSpecSettings(16, 256, 4, 4, 4, 0.7, False)
    cache = dsb.runtime.DiffSpecDraftCache(settings, max_num_reqs=4, max_model_len=64, num_kv_heads=2,
                                           head_dim=64, target_num_layers=2, dtype=torch.bfloat16,
                                           device=cuda,
                                           cos_sin_cache=torch.zeros((256, 64), device=cuda).bfloat16())
    cache.raw_key.zero_()
    cache.raw_value.zero_()
    g = torch.Generator(device="cpu").manual_seed(3)
    h = torch.randn((3, 512), generator=g).bfloat16().to(cuda)
    w = torch.randn((256, 512), generator=g).bfloat16().to(cuda)
    slots = torch.tensor([2, 0, 3], dtype=torch.int32, device=cuda)
    pos = torch.tensor([5, 63, 0], dtype=torch.int64, device=cuda)
    out = cache.project_and_write_raw(slots, pos, h, w)
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0
    for t in range(3):
        s, p = int(slots[t]), int(pos[t])
        assert torch.equal(cache.raw_key[s, p].reshape(-1), out[t, :128])
        assert torch.equal(cache.raw_value[s, p].reshape(-1), out[t, 128:])
