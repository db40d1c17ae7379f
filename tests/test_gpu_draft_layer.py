"""One Eagle3-style draft layer step (all library kernels: tcgen05 linears,
RMSNorm, RoPE, draft attention) against a torch fp32 restatement of the same
layer that rounds to bf16 at the same points (so only accumulation order
differs), at a small shape and at BASELINE config 5's layer (hidden 2048,
qkv input 4096, 32/4 heads, SwiGLU 6144, 16 tokens); and the layer's
elementwise kernels (RMSNorm, RoPE of q/k, SwiGLU) against the oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import close_bf16
from oracle import diffspec_oracle as O

pytestmark = pytest.mark.gpu


def _ref_step(layer, x_in, residual, slots, abs_pos, local_pos, wk0, wv0, cos_sin):
    """fp32 math, bf16 at the layer's rounding points; attention over the
    working cache rows [0, pos) before the step plus the new token at pos."""
    bf = torch.bfloat16
    r = lambda t: t.to(bf).float()  # noqa: E731

    def norm(x, w):  # vLLM rms_norm: the normalised value rounded before the weight
        return r(r(x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + layer.eps)) * w.float())

    def rope(x, pos):
        half = x.shape[-1] // 2
        cs = cos_sin.float()[pos.long()]
        c, s = cs[:, None, :half], cs[:, None, half:]
        return r(torch.cat((x[..., :half] * c - x[..., half:] * s, x[..., half:] * c + x[..., :half] * s), -1))

    n, hq, hk, d = x_in.shape[0], layer.hq, layer.hk, layer.d
    h = norm(x_in.float(), layer.in_norm)
    q = r(h @ layer.w_q.float().t()).view(n, hq, d)
    kv = r(h @ layer.w_kv.float().t())
    k, v = kv[:, : hk * d].view(n, hk, d), kv[:, hk * d:].view(n, hk, d)
    q, k = rope(q, local_pos), rope(k, local_pos)
    attn = torch.empty((n, hq, d), device=x_in.device)
    g = hq // hk
    for i in range(n):
        s, p = int(slots[i]), int(local_pos[i])
        K = torch.cat((wk0[s, :, :p].float(), k[i][:, None]), 1)  # [hk, p + 1, d]
        V = torch.cat((wv0[s, :, :p].float(), v[i][:, None]), 1)
        for h_ in range(hq):
            sc = (K[h_ // g] @ q[i, h_]) * d ** -0.5
            attn[i, h_] = torch.softmax(sc, 0) @ V[h_ // g]
    x = r(residual.float() + r(attn).view(n, hq * d) @ layer.w_o.float().t())  # addmm: one rounding
    gu = r(norm(x, layer.post_norm) @ layer.w_gate_up.float().t())
    act = r(r(torch.nn.functional.silu(gu[:, : layer.inter])) * gu[:, layer.inter:])  # SiluAndMul
    return r(x + act @ layer.w_down.float().t()), kv


# (hidden, qkv_in, heads, kv heads, intermediate, tokens, slots, raw length, budget):
# a small layer, and BASELINE config 5's Eagle3 layer at its decode batch of 16
_LAYER_SHAPES = {
    "small": (256, 512, 8, 1, 512, 4, 6, 600, 256),
    "config5": (2048, 4096, 32, 4, 6144, 16, 16, 4096, 2048),
}


@pytest.mark.parametrize("shape", sorted(_LAYER_SHAPES))
def test_draft_layer_step_matches_fp32_reference(dsb, cuda, shape):
    hidden, qkv_in, hq, hk, inter, n, slots_n, max_len, budget = _LAYER_SHAPES[shape]
    d = 128
    layer = dsb.draft_layer.Eagle3DraftLayer(cuda, hidden=hidden, qkv_in=qkv_in, num_heads=hq,
                                             num_kv_heads=hk, head_dim=d, intermediate=inter,
                                             seed=3)
    g = torch.Generator(device="cpu").manual_seed(11)
    bf = torch.bfloat16
    dev = lambda t: t.to(cuda)  # noqa: E731
    x_in = dev(torch.randn((n, qkv_in), generator=g)).to(bf)
    residual = dev(torch.randn((n, hidden), generator=g)).to(bf)
    slots = dev(torch.randperm(slots_n, generator=g)[:n].to(torch.int32))
    abs_pos = dev(torch.randint(budget, max_len, (n,), generator=g))
    local_pos = dev(torch.randint(2, budget, (n,), generator=g).to(torch.int32))
    local_pos[0] = budget - 1  # the last working-cache row
    raw_k = torch.zeros((slots_n, max_len, hk, d), dtype=bf, device=cuda)
    raw_v = torch.zeros_like(raw_k)
    wk = dev(torch.randn((slots_n, hk, budget, d), generator=g)).to(bf)
    wv = dev(torch.randn((slots_n, hk, budget, d), generator=g)).to(bf)
    wk0, wv0 = wk.clone(), wv.clone()
    inv = 1.0 / (1e6 ** (torch.arange(0, d, 2, dtype=torch.float64) / d))
    fr = torch.arange(budget, dtype=torch.float64)[:, None] * inv[None]
    cos_sin = dev(torch.cat((fr.cos(), fr.sin()), -1)).to(bf)
    ref, kv = _ref_step(layer, x_in, residual, slots, abs_pos, local_pos, wk0, wv0, cos_sin)
    for offset in (0, 2):  # the second step re-uses the layer's attention workspace and
        wk.copy_(wk0)       # reaches the same positions through position_offset
        wv.copy_(wv0)
        raw_k.zero_()
        raw_v.zero_()
        out = layer.step(x_in, residual, slots=slots, abs_positions=abs_pos,
                         local_positions=local_pos - offset, position_offset=offset,
                         raw_key=raw_k, raw_value=raw_v, working_key=wk, working_value=wv,
                         cos_sin=cos_sin)
        torch.cuda.synchronize()
        assert dsb._lib.read_and_clear_error_flag(cuda) == 0
        # the reference rounds to bf16 at the layer's eight rounding points, so
        # only the summation order differs: the path's bf16 tolerance holds
        close_bf16(out.float().cpu().numpy(), ref.cpu().numpy())
        for i in range(n):  # pre-RoPE K/V in the raw cache
            s, p = int(slots[i]), int(abs_pos[i])
            close_bf16(raw_k[s, p].reshape(-1).float().cpu().numpy(),
                       kv[i, : hk * d].cpu().numpy())
            close_bf16(raw_v[s, p].reshape(-1).float().cpu().numpy(),
                       kv[i, hk * d:].cpu().numpy())
        for i in range(n):  # this step's RoPE'd K and its V at its working-cache row
            s, p = int(slots[i]), int(local_pos[i])
            assert torch.equal(wk[s, :, :p], wk0[s, :, :p]) and torch.equal(wv[s, :, :p], wv0[s, :, :p])
            close_bf16(wv[s, :, p].reshape(-1).float().cpu().numpy(), kv[i, hk * d:].cpu().numpy())


_T = {"bf16": torch.bfloat16, "f16": torch.float16}
_FRAC = {"bf16": 7, "f16": 10}


def _within_one_ulp(got, ref, dtype):
    mag = np.maximum(np.abs(ref), 2.0 ** -14)
    return np.abs(got - ref) <= np.exp2(np.floor(np.log2(mag)) - _FRAC[dtype])


@pytest.mark.parametrize("dtype,rows,cols,pad", [("bf16", 16, 4096, 0), ("f16", 37, 2048, 64),
                                                 ("bf16", 1, 8, 8)])
def test_rms_norm_matches_oracle(dsb, cuda, dtype, rows, cols, pad):
    rng = np.random.default_rng(rows + cols)
    x = O.round_to(rng.standard_normal((rows, cols + pad), dtype=np.float32) * 3, dtype)
    w = O.round_to(rng.uniform(0.5, 1.5, cols).astype(np.float32), dtype)
    xt = torch.from_numpy(x).to(cuda).to(_T[dtype])[:, :cols]  # row stride cols + pad
    got = dsb.draft_layer.rms_norm(xt, torch.from_numpy(w).to(cuda).to(_T[dtype]), 1e-6)
    ref = O.rms_norm(x[:, :cols], w, 1e-6, dtype)
    g = got.float().cpu().numpy()
    assert _within_one_ulp(g, ref, dtype).all()  # fp32 sum order differs from the oracle's
    assert (g == ref).mean() > 0.99


@pytest.mark.parametrize("dtype,cs_dtype,offset", [("bf16", torch.bfloat16, 0),
                                                   ("f16", torch.float32, 0),
                                                   ("bf16", torch.bfloat16, 5)])
def test_rope_qk_matches_oracle(dsb, cuda, dtype, cs_dtype, offset):
    rng = np.random.default_rng(5)
    t_n, hq, hk, d, rows = 9, 8, 2, 128, 300
    q = O.round_to(rng.standard_normal((t_n, hq * d), dtype=np.float32), dtype)
    kv = O.round_to(rng.standard_normal((t_n, 2 * hk * d), dtype=np.float32), dtype)
    ang = np.arange(rows)[:, None] * (1e4 ** (-np.arange(d // 2) / (d // 2)))[None]
    cs = O.round_to(np.concatenate((np.cos(ang), np.sin(ang)), -1).astype(np.float32),
                    "bf16" if cs_dtype == torch.bfloat16 else "f32")
    pos = rng.integers(0, rows - offset, t_n).astype(np.int32)
    pos[3] = rows - offset  # + offset: outside the table, rows left unrotated, flagged
    dev = lambda a, tdt: torch.from_numpy(np.ascontiguousarray(a)).to(cuda).to(tdt)  # noqa: E731
    qt, kvt = dev(q, _T[dtype]), dev(kv, _T[dtype])
    k, v = dsb.draft_layer.rope_qk(qt, kvt, dev(pos, torch.int32), dev(cs, cs_dtype), hk,
                                   position_offset=offset)
    flag = dsb._lib.read_and_clear_error_flag(cuda)
    assert flag == 2  # DSB_FLAG_POSITION
    ok = np.arange(t_n) != 3
    rq, rk, rv = O.rope_qk(q[ok], kv[ok], pos[ok] + offset, cs, hk, dtype)
    np.testing.assert_array_equal(qt.float().cpu().numpy()[ok], rq)
    np.testing.assert_array_equal(k.float().cpu().numpy()[ok], rk)
    np.testing.assert_array_equal(v.float().cpu().numpy(), kv[:, hk * d:].reshape(t_n, hk, d))
    np.testing.assert_array_equal(qt.float().cpu().numpy()[3], q[3])
    np.testing.assert_array_equal(k.float().cpu().numpy()[3], kv[3, : hk * d].reshape(hk, d))


@pytest.mark.parametrize("dtype,rows,inter", [("bf16", 16, 6144), ("f16", 5, 520)])
def test_silu_mul_matches_oracle(dsb, cuda, dtype, rows, inter):
    rng = np.random.default_rng(rows)
    gu = O.round_to(rng.standard_normal((rows, 2 * inter), dtype=np.float32) * 4, dtype)
    got = dsb.draft_layer.silu_mul(torch.from_numpy(gu).to(cuda).to(_T[dtype])).float().cpu().numpy()
    ref = O.silu_mul(gu, dtype)
    assert _within_one_ulp(got, ref, dtype).all()  # fp32 exp / divide against fp64
    assert (got == ref).mean() > 0.99
