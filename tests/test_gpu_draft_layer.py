"""One Eagle3-style draft layer step (library kernels + cuBLAS GEMMs) against a
torch fp32 restatement of the same layer that rounds to bf16 at the same
points (so only accumulation order differs)."""

from __future__ import annotations

import pytest
import torch

from conftest import close_bf16

pytestmark = pytest.mark.gpu


def _ref_step(layer, x_in, residual, slots, abs_pos, local_pos, wk0, wv0, cos_sin):
    """fp32 math, bf16 at the layer's rounding points; attention over the
    working cache rows [0, pos) before the step plus the new token at pos."""
    bf = torch.bfloat16
    r = lambda t: t.to(bf).float()  # noqa: E731

    def norm(x, w):
        return r(x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + layer.eps) * w.float())

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
    x = r(residual.float() + r(attn).view(n, hq * d) @ layer.w_o.float().t())
    gu = r(norm(x, layer.post_norm) @ layer.w_gate_up.float().t())
    act = r(torch.nn.functional.silu(gu[:, : layer.inter]) * gu[:, layer.inter:])
    return r(x + act @ layer.w_down.float().t()), kv


def test_draft_layer_step_matches_fp32_reference(dsb, cuda):
    layer = dsb.draft_layer.Eagle3DraftLayer(cuda, hidden=256, qkv_in=512, num_heads=8,
                                             num_kv_heads=1, head_dim=128, intermediate=512, seed=3)
    g = torch.Generator(device="cpu").manual_seed(11)
    n, slots_n, max_len, budget = 4, 6, 600, 256
    bf = torch.bfloat16
    dev = lambda t: t.to(cuda)  # noqa: E731
    x_in = dev(torch.randn((n, 512), generator=g)).to(bf)
    residual = dev(torch.randn((n, 256), generator=g)).to(bf)
    slots = torch.tensor([4, 0, 5, 2], dtype=torch.int32, device=cuda)
    abs_pos = torch.tensor([500, 17, 320, 599], dtype=torch.int64, device=cuda)
    local_pos = torch.tensor([200, 5, 120, 255], dtype=torch.int32, device=cuda)
    raw_k = torch.zeros((slots_n, max_len, 1, 128), dtype=bf, device=cuda)
    raw_v = torch.zeros_like(raw_k)
    wk = dev(torch.randn((slots_n, 1, budget, 128), generator=g)).to(bf)
    wv = dev(torch.randn((slots_n, 1, budget, 128), generator=g)).to(bf)
    wk0, wv0 = wk.clone(), wv.clone()
    inv = 1.0 / (1e6 ** (torch.arange(0, 128, 2, dtype=torch.float64) / 128))
    fr = torch.arange(budget, dtype=torch.float64)[:, None] * inv[None]
    cos_sin = dev(torch.cat((fr.cos(), fr.sin()), -1)).to(bf)
    for _ in range(2):  # the second step re-uses the layer's attention workspace
        wk.copy_(wk0)
        wv.copy_(wv0)
        out = layer.step(x_in, residual, slots=slots, abs_positions=abs_pos,
                         local_positions=local_pos, raw_key=raw_k, raw_value=raw_v,
                         working_key=wk, working_value=wv, cos_sin=cos_sin)
        torch.cuda.synchronize()
        assert dsb._lib.read_and_clear_error_flag(cuda) == 0
        ref, kv = _ref_step(layer, x_in, residual, slots, abs_pos, local_pos, wk0, wv0, cos_sin)
        # eight bf16 rounding points in the layer, each of which can round one
        # ulp apart when only the summation order differs: mean 5e-3 relative
        close_bf16(out.float().cpu().numpy(), ref.cpu().numpy(), mean_rel=5e-3)
        for i in range(n):  # pre-RoPE K/V in the raw cache
            s, p = int(slots[i]), int(abs_pos[i])
            close_bf16(raw_k[s, p].reshape(-1).float().cpu().numpy(), kv[i, :128].cpu().numpy())
            close_bf16(raw_v[s, p].reshape(-1).float().cpu().numpy(), kv[i, 128:].cpu().numpy())
