"""Stand-in for vllm_ascend.ops.triton.rope.rope_forward_triton_siso.

The reference calls this third-party kernel in place on [tokens, heads, dim]
K rows at the given positions (diffspec/kernels.py:203-209).  Its source is
not vendored, so this restates the published rotary-embedding math with fp32
compute (x1*cos - x2*sin, x2*cos + x1*sin; NeoX halves or GPT-J pairs) and
rounds once to the tensor dtype.
"""

import torch


def rope_forward_triton_siso(x, *, cos_sin_cache, positions, rope_dim, is_neox_style):
    if rope_dim == 0:
        return x
    half = rope_dim // 2
    cs = cos_sin_cache.index_select(0, positions.long()).float()
    cos = cs[:, None, :half]
    sin = cs[:, None, half:rope_dim]
    rot = x[..., :rope_dim].float()
    if is_neox_style:
        first, second = rot[..., :half], rot[..., half:]
        out = torch.cat((first * cos - second * sin, second * cos + first * sin), dim=-1)
    else:
        first, second = rot[..., 0::2], rot[..., 1::2]
        out = torch.stack((first * cos - second * sin, second * cos + first * sin), dim=-1).flatten(-2)
    x[..., :rope_dim] = out.to(x.dtype)
    return x
