"""One Eagle3-style draft decoder layer over the DiffSpec draft cache.

The draft model of diffspec runs one decoder layer per draft step: its qkv
projection takes the token embedding concatenated with the target's hidden
state (diffspec/vllm_patch.py:189-225), the sink op hands the pre-RoPE K/V
to the canonical cache (vllm_patch.py:132-178, runtime.py:1602-1618), RoPE is
applied at the working cache's local positions (runtime.py:1767-1794), and
the attention runs over the compact working cache (runtime.py:2024-2134),
followed by the output projection and a SwiGLU MLP with RMSNorm.

Here the K/V projection, the raw-cache write and the draft attention are this
library's kernels (``kv_projection_write_raw``, ``draft_decode_attention``);
the query / output projections and the MLP are plain GEMMs (cuBLAS through
torch) and the norms, RoPE and activation are torch elementwise ops.  The
weights are random (no checkpoint is involved); the layer exists to turn the
kernels into draft tokens per second and to show how the
pieces compose.  The LM head is not included: its vocabulary is unspecified.
"""

from __future__ import annotations

import torch

from .attention import AttentionWorkspace, draft_decode_attention
from .kernels import kv_projection_write_raw

__all__ = ["Eagle3DraftLayer", "rope_neox"]


def rope_neox(x: torch.Tensor, cos_sin: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
    """NeoX rotation of ``x [n, heads, D]`` at ``positions [n]`` with a
    ``[cos | sin]`` table (fp32 math, one rounding)."""
    half = x.shape[-1] // 2
    cs = cos_sin.index_select(0, positions.long()).float()
    cos, sin = cs[:, None, :half], cs[:, None, half:]
    xf = x.float()
    x1, x2 = xf[..., :half], xf[..., half:]
    return torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), -1).to(x.dtype)


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * weight.float()).to(x.dtype)


class Eagle3DraftLayer:
    """Random-init weights of one draft layer (bf16): hidden 2048, qkv input
    4096 (embedding + hidden), 32 query / 4 kv heads of 128, SwiGLU 6144."""

    def __init__(self, device, *, hidden=2048, qkv_in=4096, num_heads=32, num_kv_heads=4,
                 head_dim=128, intermediate=6144, dtype=torch.bfloat16, seed=0, eps=1e-6):
        g = torch.Generator(device=device).manual_seed(seed)

        def w(rows, cols):
            return (torch.randn((rows, cols), generator=g, device=device) / cols ** 0.5).to(dtype)

        self.hq, self.hk, self.d, self.eps = num_heads, num_kv_heads, head_dim, eps
        self.inter = intermediate
        self.w_q = w(num_heads * head_dim, qkv_in)
        self.w_kv = w(2 * num_kv_heads * head_dim, qkv_in)  # K rows, then V rows
        self.w_o = w(hidden, num_heads * head_dim)
        self.w_gate_up = w(2 * intermediate, hidden)
        self.w_down = w(hidden, intermediate)
        self.in_norm = torch.ones(qkv_in, dtype=dtype, device=device)
        self.post_norm = torch.ones(hidden, dtype=dtype, device=device)
        self.workspace = AttentionWorkspace(device)

    def weight_bytes(self) -> int:
        return sum(t.numel() * t.element_size()
                   for t in (self.w_q, self.w_kv, self.w_o, self.w_gate_up, self.w_down))

    def step(self, x_in, residual, *, slots, abs_positions, local_positions, raw_key, raw_value,
             working_key, working_value, cos_sin, out=None):
        """One draft step for ``n`` rows: ``x_in [n, qkv_in]`` (embedding +
        hidden), ``residual [n, hidden]``.  Writes this step's pre-RoPE K/V to
        the raw caches at ``[slots, abs_positions]`` and its RoPE'd K/V into
        the working caches at ``local_positions``; returns the layer output
        ``[n, hidden]``."""
        n = x_in.shape[0]
        h = rms_norm(x_in, self.in_norm, self.eps)
        q = (h @ self.w_q.t()).view(n, self.hq, self.d)
        kv = kv_projection_write_raw(h, self.w_kv, slots, abs_positions, raw_key, raw_value)
        k = kv[:, : self.hk * self.d].view(n, self.hk, self.d)
        v = kv[:, self.hk * self.d:].view(n, self.hk, self.d)
        q = rope_neox(q, cos_sin, local_positions)
        k = rope_neox(k, cos_sin, local_positions)
        attn = draft_decode_attention(q, k, v, working_key, working_value, slots, local_positions,
                                      self.d ** -0.5, workspace=self.workspace)
        x = residual + attn.view(n, self.hq * self.d) @ self.w_o.t()
        gu = rms_norm(x, self.post_norm, self.eps) @ self.w_gate_up.t()
        act = torch.nn.functional.silu(gu[:, : self.inter].float()) * gu[:, self.inter:].float()
        return x + act.to(x.dtype) @ self.w_down.t()
