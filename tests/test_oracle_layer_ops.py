"""The oracle's draft-layer elementwise stages (RMSNorm, SwiGLU, RoPE of one
step) against torch fp32 statements of the same formulas, and the host-side
validation of the library wrappers (no GPU)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import diffspec_oracle as O


def test_rms_norm_and_silu_mul_agree_with_torch():
    rng = np.random.default_rng(0)
    x = O.round_to(rng.standard_normal((6, 256), dtype=np.float32), "bf16")
    w = O.round_to(rng.uniform(0.5, 1.5, 256).astype(np.float32), "bf16")
    xt = torch.from_numpy(x)
    ref = ((xt * torch.rsqrt(xt.pow(2).mean(-1, keepdim=True) + 1e-6)).bfloat16().float()
           * torch.from_numpy(w)).bfloat16()
    got = O.rms_norm(x, w, 1e-6)
    assert (got == ref.float().numpy()).mean() > 0.99
    assert np.abs(got - ref.float().numpy()).max() <= 2.0 ** -6 * np.abs(got).max()
    gu = O.round_to(rng.standard_normal((6, 64), dtype=np.float32) * 4, "bf16")
    gt = torch.from_numpy(gu)
    ref = (torch.nn.functional.silu(gt[:, :32]).bfloat16().float() * gt[:, 32:]).bfloat16().float().numpy()
    got = O.silu_mul(gu)
    assert (got == ref).mean() > 0.99


def test_rope_qk_rotates_queries_and_keys_and_passes_values():
    rng = np.random.default_rng(1)
    t_n, hq, hk, d = 3, 4, 2, 8
    q = O.round_to(rng.standard_normal((t_n, hq * d), dtype=np.float32), "bf16")
    kv = O.round_to(rng.standard_normal((t_n, 2 * hk * d), dtype=np.float32), "bf16")
    ang = np.arange(10)[:, None] * (1e4 ** (-np.arange(d // 2) / (d // 2)))[None]
    cs = np.concatenate((np.cos(ang), np.sin(ang)), -1).astype(np.float32)
    pos = np.array([0, 4, 9])
    rq, rk, rv = O.rope_qk(q, kv, pos, cs, hk)
    np.testing.assert_array_equal(rq[0], q[0])  # position 0: identity
    np.testing.assert_array_equal(rv, kv[:, hk * d:].reshape(t_n, hk, d))
    # rotation keeps the norm of each (i, i + half) pair
    kk = kv[:, : hk * d].reshape(t_n, hk, d)
    np.testing.assert_allclose(rk[..., :4] ** 2 + rk[..., 4:] ** 2, kk[..., :4] ** 2 + kk[..., 4:] ** 2,
                               rtol=3e-2, atol=1e-3)


def test_layer_op_wrappers_reject_host_tensors(dsb):
    x = torch.zeros((2, 16), dtype=torch.bfloat16)
    with pytest.raises((ValueError, RuntimeError)):
        dsb.draft_layer.rms_norm(x, torch.ones(16, dtype=torch.bfloat16), 1e-6)
    with pytest.raises(ValueError):
        dsb.draft_layer.rms_norm(x, torch.ones(8, dtype=torch.bfloat16), 1e-6)
    with pytest.raises((ValueError, RuntimeError)):
        dsb.draft_layer.silu_mul(torch.zeros((2, 32), dtype=torch.bfloat16))
    with pytest.raises(ValueError):
        dsb.draft_layer.rope_qk(torch.zeros((2, 16), dtype=torch.bfloat16),
                                torch.zeros((2, 16), dtype=torch.bfloat16),
                                torch.zeros(2, dtype=torch.int64), torch.zeros((4, 8)), 1)


_FRAC = {"bf16": 7, "f16": 10}


def _ulp(a, dtype):
    return np.exp2(np.floor(np.log2(np.maximum(np.abs(a), 2.0 ** -14))) - _FRAC[dtype])


@pytest.mark.parametrize("case", ["rms_bf16", "rms_f16", "silu_bf16", "silu_f16"])
def test_oracle_matches_vllm_golden_vectors(case):
    """tests/golden/layer_ops.npz holds vLLM's own rms_norm / SiluAndMul
    outputs (tests/golden/make_layer_golden.py)."""
    from conftest import ROOT
    g = np.load(ROOT / "tests" / "golden" / "layer_ops.npz")
    dtype = case.split("_")[1]
    x, y = g[f"{case}_x"], g[f"{case}_y"]
    if case.startswith("rms"):
        got = O.rms_norm(x, g[f"{case}_w"], float(g["eps"]), dtype)
    else:
        got = O.silu_mul(x, dtype)
    # same rounding points; only the fp32 reduction / exp of vLLM's torch ops
    # can put a value on the other side of a rounding boundary
    assert (np.abs(got - y) <= _ulp(y, dtype)).all()
    assert (got == y).mean() > 0.99


def test_causal_row_lengths_of_target_spans(dsb):
    """Each query row of a target pass sees its request's prefix up to itself."""
    f = dsb.runtime.causal_row_lengths
    assert f([3, 6], [300, 150]) == ([298, 299, 300, 148, 149, 150], [0, 0, 0, 1, 1, 1])
    assert f([1, 2], [7, 5]) == ([7, 5], [0, 1])          # plain decode: one row each
    assert f([2, 2, 4], [1, 9, 3]) == ([0, 1, 2, 3], [0, 0, 2, 2])  # empty span; short prefix
    with pytest.raises(ValueError):
        f([3, 2], [5, 5])
    with pytest.raises(ValueError):
        f([1, 2, 3], [5, 5])


def test_oracle_target_lse_reproduces_the_scores_own_lse():
    """oracle.paged_decode_attention_lse's LSE, given to the chunk scores,
    gives the scores whose LSE they compute themselves (the softmax_lse=None
    branch, pinned to the reference's fixtures), and its output is the
    softmax-weighted V."""
    rng = np.random.default_rng(8)
    rows, hq, hk, bs, d = 3, 8, 2, 16, 128
    lens = np.array([100, 37, 64])
    table = rng.permutation(3 * 7).reshape(3, 7).astype(np.int32)
    kc = O.round_to(rng.standard_normal((21, bs, hk, d), dtype=np.float32), "bf16")
    vc = O.round_to(rng.standard_normal((21, bs, hk, d), dtype=np.float32), "bf16")
    q = O.round_to(rng.standard_normal((rows, hq, d), dtype=np.float32), "bf16")
    out, lse = O.paged_decode_attention_lse(q, kc, vc, table, lens, d ** -0.5, dtype="f32")
    with_lse = O.paged_chunk_attention_scores(q, kc, lse, table, lens, 16, 112, d ** -0.5)
    own = O.paged_chunk_attention_scores(q, kc, None, table, lens, 16, 112, d ** -0.5)
    np.testing.assert_allclose(with_lse, own, rtol=1e-5, atol=1e-9)
    # row 1, head 3 by hand
    toks = np.arange(37)
    k = kc[table[1][toks // bs], toks % bs, 3 // 4].astype(np.float64)
    v = vc[table[1][toks // bs], toks % bs, 3 // 4].astype(np.float64)
    s = k @ q[1, 3].astype(np.float64) * d ** -0.5
    p = np.exp(s - s.max())
    np.testing.assert_allclose(out[1, 3], p @ v / p.sum(), rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(lse[1, 3], s.max() + np.log(p.sum()), rtol=1e-6)


def test_target_attention_wrapper_rejects_bad_arguments(dsb):
    f = dsb.kernels.paged_decode_attention_lse
    q = torch.zeros((2, 8, 128), dtype=torch.bfloat16)
    kc = torch.zeros((4, 16, 2, 128), dtype=torch.bfloat16)
    bt = torch.zeros((2, 2), dtype=torch.int32)
    lens = torch.ones(2, dtype=torch.int32)
    with pytest.raises(ValueError, match="table_rows"):
        f(q, kc, kc, bt, lens, scale=0.1, max_seq_len=32, table_rows=torch.zeros(1, dtype=torch.int32))
    with pytest.raises(ValueError, match="max_seq_len"):
        f(q, kc, kc, bt, lens, scale=0.1, max_seq_len=-1)
    # tokens_per_split <= 0 picks the library's default of 512, in the wrapper
    # (which then only fails on the CPU tensors) and in the C ABI alike
    with pytest.raises(ValueError, match="CUDA"):
        f(q, kc, kc, bt, lens, scale=0.1, max_seq_len=32, tokens_per_split=0)
    lib = dsb._lib.load()
    assert lib.dsb_paged_decode_scratch_floats(2, 8, 4096, 0) == \
        lib.dsb_paged_decode_scratch_floats(2, 8, 4096, 512) == 2 * 8 * 8 * 130
    with pytest.raises(ValueError):
        f(q, kc[..., :64], kc[..., :64], bt, lens, scale=0.1, max_seq_len=32)  # head dims differ
    with pytest.raises(ValueError):
        f(q, kc, kc, bt, lens[:1], scale=0.1, max_seq_len=32)  # seq_lens short
