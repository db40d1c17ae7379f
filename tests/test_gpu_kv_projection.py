"""Draft-layer K/V projection with the raw-cache write in its epilogue
(dsb_kv_projection_write_raw, dsb_qkv_projection_write_raw) and the
draft-layer linear with its plain / residual / SwiGLU epilogues
(dsb_draft_linear) against the oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import diffspec_oracle as O

pytestmark = pytest.mark.gpu

_T = {"bf16": torch.bfloat16, "f16": torch.float16}


@pytest.fixture(autouse=True, params=["auto", "ranks16", "ranks8", "ranks1"])
def cluster_size(request, monkeypatch):
    """Every case with the split-K cluster size chosen per launch and with it
    forced to 16, 8 (DSB_KV_PROJECTION_RANKS8=1) and 1 (DSB_LINEAR_RANKS)."""
    if request.param == "ranks8":
        monkeypatch.setenv("DSB_KV_PROJECTION_RANKS8", "1")
    elif request.param != "auto":
        monkeypatch.setenv("DSB_LINEAR_RANKS", request.param[5:])
    return request.param
_FRAC = {"bf16": 7, "f16": 10}  # fraction bits of the stored type


def within_one_ulp(got, ref_f32, dtype, k=0):
    """|got - ref| <= one unit in the last place of the stored type at |ref|
    (the fp32 sums differ only in order from the oracle's), or, for outputs
    near zero whose ulp is below the fp32 summation error of k unit-scale
    products, <= sqrt(k) * 2^-20 (about 16x that error's typical size)."""
    mag = np.maximum(np.abs(ref_f32), 2.0 ** -14)
    ulp = np.exp2(np.floor(np.log2(mag)) - _FRAC[dtype])
    return np.abs(got - ref_f32) <= np.maximum(ulp, np.sqrt(k) * 2.0 ** -20)


@pytest.mark.parametrize("dtype,tokens,hidden,hk,d", [
    ("bf16", 16, 4096, 4, 128),   # config-5 decode step: Eagle3 qkv input 4096, 4 kv heads
    ("bf16", 37, 512, 2, 64),     # three token tiles, ragged last one
    ("f16", 5, 1024, 1, 128),     # fewer tokens than a tile, ranks with one k-block each
    ("bf16", 20, 256, 4, 128),    # fewer k-blocks than cluster ranks
    ("bf16", 16, 6144, 4, 128),   # more k-blocks per rank than ring slots
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
    assert within_one_ulp(got, ref_f32, dtype, hidden).all()
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


def _cells(rng, tokens, slots_n, max_len):
    slots = (np.arange(tokens) % slots_n).astype(np.int32)
    positions = (np.arange(tokens) // slots_n * 7 + 2).astype(np.int64) % max_len
    return slots, positions


@pytest.mark.parametrize("prefetch", [False, True])
@pytest.mark.parametrize("tokens,hidden,qf,hk,d", [(16, 4096, 4096, 4, 128), (21, 1024, 256, 1, 128)])
def test_qkv_projection_routes_query_and_kv(dsb, cuda, prefetch, tokens, hidden, qf, hk, d):
    rng = np.random.default_rng(hidden + qf)
    slots_n, max_len = 8, 64
    h = O.round_to(rng.standard_normal((tokens, hidden), dtype=np.float32), "bf16")
    w = O.round_to(rng.standard_normal((qf + 2 * hk * d, hidden), dtype=np.float32) / np.sqrt(hidden),
                   "bf16")
    slots, positions = _cells(rng, tokens, slots_n, max_len)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    rk = torch.zeros((slots_n, max_len, hk, d), dtype=torch.bfloat16, device=cuda)
    rv = torch.zeros_like(rk)
    q, kv = dsb.kernels.qkv_projection_write_raw(dev(h).bfloat16(), dev(w).bfloat16(), qf,
                                                 dev(slots), dev(positions), rk, rv,
                                                 prefetch_weight=prefetch)
    torch.cuda.synchronize()
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0
    ref = h.astype(np.float64) @ w.astype(np.float64).T
    got = torch.cat((q, kv), 1).float().cpu().numpy()
    assert within_one_ulp(got, ref, "bf16", hidden).all()
    assert (got == O.linear(h, w)).mean() > 0.99
    half = hk * d
    for t in range(tokens):
        np.testing.assert_array_equal(rk[slots[t], positions[t]].reshape(-1).float().cpu().numpy(),
                                      got[t, qf: qf + half])
        np.testing.assert_array_equal(rv[slots[t], positions[t]].reshape(-1).float().cpu().numpy(),
                                      got[t, qf + half:])


@pytest.mark.parametrize("epilogue", ["plain", "residual", "swiglu"])
@pytest.mark.parametrize("dtype,tokens,k,rows", [
    ("bf16", 16, 4096, 2048),    # config-5 o_proj shape
    ("bf16", 16, 2048, 1024),    # gate_up-like (inter 512)
    ("f16", 37, 6144, 256),      # down_proj K: ring refills; ragged token tiles
    ("bf16", 3, 64, 128),        # one k-block: most ranks have none
])
def test_draft_linear_epilogues_match_oracle(dsb, cuda, epilogue, dtype, tokens, k, rows):
    rng = np.random.default_rng(tokens * 7 + k + rows)
    x = O.round_to(rng.standard_normal((tokens, k), dtype=np.float32), dtype)
    w = O.round_to(rng.standard_normal((rows, k), dtype=np.float32) / np.sqrt(k), dtype)
    tdt = _T[dtype]
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda).to(tdt)  # noqa: E731
    dl = dsb.draft_layer
    if epilogue == "swiglu":
        got = dl.draft_linear(dev(x), dl.interleave_gate_up(dev(w)), "swiglu").float().cpu().numpy()
        torch.cuda.synchronize()
        gu = O.linear(x, w, dtype=dtype)
        ref = O.silu_mul(gu, dtype)
        # gate and up are rounded sums, each of which may round one ulp away
        # from the oracle's (summation order; more near zero): bound = what
        # that moves silu(gate) * up by, plus two ulp of the output
        def ulp(a):
            return np.exp2(np.floor(np.log2(np.maximum(np.abs(a), 2.0 ** -14))) - _FRAC[dtype])
        inter = rows // 2
        g, u = gu[:, :inter].astype(np.float64), gu[:, inter:].astype(np.float64)
        sig = 1.0 / (1.0 + np.exp(-g))
        floor = np.sqrt(k) * 2.0 ** -20  # fp32 summation error near zero (within_one_ulp)
        err_g, err_u = np.maximum(ulp(g), floor), np.maximum(ulp(u), floor)
        bound = (np.abs(sig * (1 + g * (1 - sig))) * err_g * np.abs(u) + np.abs(g * sig) * err_u
                 + ulp(g * sig) * np.abs(u) + 2 * ulp(ref))  # + the rounded silu's own ulp
        assert (np.abs(got - ref) <= bound).all()
        # two rounded inputs per output: 0.955 equal seen with one unsplit fp16
        # accumulator over K = 6144, > 0.99 with split ones
        assert (got == ref).mean() > 0.94
    else:
        res = O.round_to(rng.standard_normal((tokens, rows), dtype=np.float32), dtype)
        got = dl.draft_linear(dev(x), dev(w), epilogue,
                              residual=dev(res) if epilogue == "residual" else None)
        got = got.float().cpu().numpy()
        ref64 = x.astype(np.float64) @ w.astype(np.float64).T
        if epilogue == "residual":
            ref64 = ref64 + res
        assert within_one_ulp(got, ref64, dtype, k).all()
        # one unsplit accumulator over K = 6144 (forced 1-CTA clusters) rounds
        # fp16 outputs away from the oracle's sequential fp32 sum slightly more often
        same = (got == O.linear(x, w, res if epilogue == "residual" else None, dtype)).mean()
        assert same > 0.97
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0


@pytest.mark.parametrize("rows,k", [(5120, 4096), (2048, 4096), (12288, 2048), (2048, 6144),
                                    (256, 128)])
def test_packed_weight_is_bit_identical(dsb, cuda, rows, k):
    """Tile-packed weights (pack_linear_weight) give the same bits as the
    row-major weight in every epilogue and in the q / K-V routing with the
    raw-cache write: the kernel reads the same 128 x 64 blocks in the same
    order, only from contiguous runs."""
    g = torch.Generator(device=cuda).manual_seed(rows + k)
    dl = dsb.draft_layer
    w = (torch.randn((rows, k), generator=g, device=cuda) / k ** 0.5).bfloat16()
    x = torch.randn((16, k), generator=g, device=cuda).bfloat16()
    res = torch.randn((16, rows), generator=g, device=cuda).bfloat16()
    wp = dl.pack_linear_weight(w)
    blocks = w.view(rows // 128, 128, k // 64, 8, 8).permute(0, 2, 1, 3, 4)  # [m, kb, r, p, 8]
    swz = (torch.arange(8, device=cuda)[None, :] ^ torch.arange(128, device=cuda)[:, None] % 8)
    expect = torch.empty_like(blocks)
    expect[:, :, torch.arange(128, device=cuda)[:, None], swz] = blocks  # piece p at p ^ (r % 8)
    assert torch.equal(wp.view(rows // 128, k // 64, 128, 8, 8), expect)
    for epi in ("plain", "residual"):
        r = res if epi == "residual" else None
        assert torch.equal(dl.draft_linear(x, w, epi, residual=r),
                           dl.draft_linear(x, wp, epi, residual=r, packed=True))
    if rows % 256 == 0:
        wt = dl.interleave_gate_up(w)
        assert torch.equal(dl.draft_linear(x, wt, "swiglu"),
                           dl.draft_linear(x, dl.pack_linear_weight(wt), "swiglu", packed=True))
    # the L2 prefetch of the rest of the weight only moves data earlier
    for weight, packed in ((w, False), (wp, True)):
        assert torch.equal(dl.draft_linear(x, weight, "residual", residual=res, packed=packed),
                           dl.draft_linear(x, weight, "residual", residual=res, packed=packed,
                                           prefetch_l2=True))
    if rows == 5120:  # the config-5 qkv projection: 32 query heads + 4 kv heads of 128
        rk = torch.zeros((16, 64, 4, 128), dtype=torch.bfloat16, device=cuda)
        outs = []
        for weight, packed, l2 in ((w, False, False), (wp, True, False), (wp, True, True),
                                   (w, False, True)):
            rk_, rv_ = rk.clone(), rk.clone()
            q, kv = dsb.kernels.qkv_projection_write_raw(
                x, weight, 4096, torch.arange(16, dtype=torch.int32, device=cuda),
                torch.arange(16, dtype=torch.int64, device=cuda), rk_, rv_, packed_weight=packed,
                prefetch_weight=l2, prefetch_l2=l2)
            outs.append((q, kv, rk_, rv_))
        for other in outs[1:]:
            for a, b in zip(outs[0], other):
                assert torch.equal(a, b)
    torch.cuda.synchronize()
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0
