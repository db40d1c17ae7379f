"""Deterministic inputs of the golden fixtures, shared by make_golden.py and
the tests.

Inputs are drawn from numpy's PCG64 generator, whose streams are identical
across platforms for a given numpy version; every fixture stores a CRC32 of
the inputs it was generated from and the tests check it before comparing, so
a change of generator cannot pass silently.  Floating-point inputs are rounded
to their storage dtype here (bf16 / fp16 values held in float32 arrays).
"""

from __future__ import annotations

import zlib

import numpy as np

from oracle.diffspec_oracle import round_to


def rng(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(seed))


def normal(g: np.random.Generator, shape, dtype: str) -> np.ndarray:
    return round_to(g.standard_normal(shape, dtype=np.float32), dtype)


def crc(*arrays: np.ndarray) -> int:
    h = 0
    for a in arrays:
        h = zlib.crc32(np.ascontiguousarray(a).tobytes(), h)
    return h


def cos_sin_table(positions: int, rotary_dim: int, theta: float = 1.0e6) -> np.ndarray:
    """[cos | sin] table with inv_freq = theta^(-2i/d) (vLLM's RoPE table layout)."""
    inv = 1.0 / (theta ** (np.arange(0, rotary_dim, 2, dtype=np.float64) / rotary_dim))
    freqs = np.arange(positions, dtype=np.float64)[:, None] * inv[None, :]
    return np.concatenate([np.cos(freqs), np.sin(freqs)], axis=-1).astype(np.float32)


# ---------------------------------------------------------------- scores (A1/A2)
SCORE_CASES = [
    # block_size, Hq, Hk, chunk, D, lengths, dtype
    (64, 4, 1, 16, 128, [2 * 64 + 13, 64 + 25], "bf16"),
    (16, 8, 2, 64, 128, [300, 77, 1], "bf16"),
    (128, 6, 1, 32, 64, [500, 129], "bf16"),
    (64, 12, 2, 16, 256, [200, 64], "bf16"),
    (16, 32, 4, 64, 128, [700, 300, 0], "bf16"),
    (32, 8, 1, 32, 128, [257], "f16"),
    (8, 4, 2, 8, 32, [50, 13], "f32"),
    (48, 16, 2, 32, 128, [333, 96], "bf16"),
]


def scores_inputs(i: int) -> dict:
    bs, hq, hk, c, d, lengths, dtype = SCORE_CASES[i]
    g = rng(1000 + i)
    b = len(lengths)
    max_len = max(lengths)
    pages = max(1, (max_len + bs - 1) // bs)
    nblocks = b * pages + 3
    query = normal(g, (b, hq, d), dtype)
    keys = normal(g, (nblocks, bs, hk, d), dtype)
    table = g.permutation(nblocks)[: b * pages].reshape(b, pages).astype(np.int32)
    return dict(block_size=bs, hq=hq, hk=hk, chunk=c, d=d, lengths=np.array(lengths, np.int32),
                dtype=dtype, query=query, key_cache=keys, block_table=table, max_len=max_len,
                scale=d ** -0.5)


def dense_lse(inp: dict) -> np.ndarray:
    """Per-(row, query head) log-sum-exp over the row's tokens (fp64)."""
    q, kc, bt = inp["query"], inp["key_cache"], inp["block_table"]
    b, hq, d = q.shape
    hk, bs = inp["hk"], inp["block_size"]
    lse = np.zeros((b, hq), dtype=np.float64)
    for r, length in enumerate(inp["lengths"]):
        if length == 0:
            continue
        tok = np.arange(length)
        keys = kc[bt[r][tok // bs], tok % bs].astype(np.float64)
        logits = np.einsum("kgd,tkd->kgt", q[r].astype(np.float64).reshape(hk, hq // hk, d), keys)
        logits = logits.reshape(hq, length) * inp["scale"]
        m = logits.max(axis=1, keepdims=True)
        lse[r] = (m + np.log(np.exp(logits - m).sum(axis=1, keepdims=True)))[:, 0]
    return lse.astype(np.float32)


# ---------------------------------------------------------------- select (A4)
def select_cases() -> list[tuple[int, int, int]]:
    g = rng(23)
    cases = []
    for c in (16, 32, 64):
        for max_chunks in (1, 2, 8, 31):
            for n in (1, 5, max_chunks, max_chunks + 1, 100, 640):
                partial = int(g.integers(0, 2))
                seq_len = n * c - (int(g.integers(1, c)) if partial else 0)
                cases.append((seq_len, c, max_chunks * c))
    return cases


def select_scores(i: int, n: int) -> np.ndarray:
    return rng(5000 + i).random(n, dtype=np.float32)


# ---------------------------------------------------------------- rebuild (A6)
REBUILD_CASES = [
    # heads, dim, rotary_dim, neox, slots
    (2, 128, 128, True, [0, 1]),
    (2, 128, 128, True, [2, 0]),
    (4, 256, 256, True, [0, 1]),
    (4, 256, 128, True, [2, 0]),
    (2, 128, 64, False, [0, 1]),
    (4, 64, 64, False, [2, 0]),
]
REBUILD_ENDS = (0, 1, 7, 62, 66, 73)
REBUILD_CHUNK, REBUILD_BUDGET, REBUILD_DEPTH, REBUILD_SLOTS, REBUILD_LEN = 8, 64, 4, 3, 128


def rebuild_inputs(ci: int) -> dict:
    heads, dim, rot, neox, slots = REBUILD_CASES[ci]
    g = rng(1700 + ci)
    shape = (REBUILD_SLOTS, REBUILD_LEN, heads, dim)
    return dict(raw_key=normal(g, shape, "bf16"), raw_value=normal(g, shape, "bf16"),
                cos_sin=round_to(cos_sin_table(128, rot), "bf16"), heads=heads, dim=dim, rot=rot,
                neox=neox, slots=slots)


# ---------------------------------------------------------------- gather (A7)
GATHER_CASES = [(16, 2, 128, 128, True), (64, 4, 64, 32, False), (8, 1, 256, 128, True)]
GATHER_TOKENS = 24


def gather_inputs(i: int) -> dict:
    bs, heads, dim, rot, neox = GATHER_CASES[i]
    g = rng(4000 + i)
    nblocks = 12
    raw_k = normal(g, (nblocks, bs, heads, dim), "bf16")
    raw_v = normal(g, (nblocks, bs, heads, dim), "bf16")
    table = g.permutation(nblocks)[:8].reshape(2, 4).astype(np.int32)
    sel = g.integers(0, 4 * bs, size=(2, GATHER_TOKENS)).astype(np.int64)
    sel[0, -3:] = -1
    sel[1, 5] = -1
    return dict(block_size=bs, heads=heads, dim=dim, rot=rot, neox=neox, raw_key=raw_k,
                raw_value=raw_v, block_table=table, selected=sel,
                cos_sin=round_to(cos_sin_table(64, rot), "bf16"))


# ---------------------------------------------------------------- attention (A8)
def attention_cases() -> list[tuple[int, int, int, int, list[int]]]:
    cases = []
    for heads, dim, qheads, budget in ((2, 128, 8, 64), (4, 128, 32, 512), (1, 64, 8, 256),
                                        (2, 128, 32, 256), (4, 256, 4, 64)):
        for slots in ([0], [0, 1, 2], [3, 0, 2]):
            cases.append((heads, dim, qheads, budget, slots))
    return cases


ATTN_ROWS = 5  # query rows per step; rows past len(slots) are graph padding


def attention_inputs(i: int) -> dict:
    heads, dim, qheads, budget, slots = attention_cases()[i]
    g = rng(3100 + i)
    shape = (4, heads, budget, dim)
    base = [3, 11, 6] if budget <= 64 else [3, budget - 70, budget // 3]
    steps = []
    for _ in range(2):
        steps.append(dict(query=normal(g, (ATTN_ROWS, qheads, dim), "bf16"),
                          key=normal(g, (ATTN_ROWS, heads, dim), "bf16"),
                          value=normal(g, (ATTN_ROWS, heads, dim), "bf16")))
    return dict(heads=heads, dim=dim, qheads=qheads, budget=budget, slots=slots,
                working_key=normal(g, shape, "bf16"), working_value=normal(g, shape, "bf16"),
                positions=base[: len(slots)], steps=steps)


# ---------------------------------------------------------------- retrieval hook (A3)
HOOK_CASES = [(counts, padding) for counts in ([1, 2], [4, 4], [0, 2], [0, 0], [3, 1])
              for padding in (False, True)]
HOOK_CHUNK, HOOK_BUDGET, HOOK_HQ, HOOK_HK, HOOK_D, HOOK_BS = 4, 32, 4, 1, 64, 16


def hook_inputs(i: int) -> dict:
    counts, padding = HOOK_CASES[i]
    g = rng(9000 + i)
    rows = 3 if padding else 2
    query = normal(g, (4 * rows, HOOK_HQ, HOOK_D), "bf16")
    lse = (g.random((4 * rows, HOOK_HQ), dtype=np.float32) * 3 + 4).astype(np.float32)
    key_cache = normal(g, (20, HOOK_BS, HOOK_HK, HOOK_D), "bf16")
    tables = np.array([[0, 1, 2, 3, 4, 5], [6, 7, 8, 9, 10, 11], [12, 13, 14, 15, 16, 17]][:rows],
                      dtype=np.int32)
    return dict(counts=np.array(counts, np.int64), rows=rows, query=query, lse=lse,
                key_cache=key_cache, block_tables=tables,
                seq_lens=np.array([90, 70, 1][:rows], np.int32),
                query_ends=np.array([4 * (r + 1) for r in range(rows)], np.int32))


# ---------------------------------------------------------------- config 1 chain (A2, A4-A6, A8)
# one request, 4096 tokens, chunk 32, budget 512, 1 kv head
# + 8 query heads of 128, fp32, RoPE theta 1e6, K = 4 draft tokens with the
# last 3 rejected (retrieval over 4093 tokens, history ending at 4092).  The
# keys of 4 planted chunks are the committed query's GQA-group mean + N(0,
# 0.1).  Values are drawn exact in bf16 so the GPU path (bf16 caches) sees
# the same numbers as the reference's fp32 run.  The target's keys double as
# the draft's pre-RoPE raw keys.
CONFIG1 = dict(tokens=4096, chunk=32, budget=512, window=128, hk=1, hq=8, d=128, theta=1e6,
               depth=4, rejected=3, planted=(10, 40, 77, 100))


def config1_inputs() -> dict:
    c = CONFIG1
    g = rng(1001)
    t, hk, hq, d = c["tokens"], c["hk"], c["hq"], c["d"]
    keys = normal(g, (t, hk, d), "bf16")
    values = normal(g, (t, hk, d), "bf16")
    query = normal(g, (hq, d), "bf16")
    mean = query.reshape(hk, hq // hk, d).mean(1)
    for ch in c["planted"]:
        noise = 0.1 * g.standard_normal((c["chunk"], hk, d)).astype(np.float32)
        keys[ch * c["chunk"]:(ch + 1) * c["chunk"]] = round_to(mean[None] + noise, "bf16")
    steps = dict(query=normal(g, (c["depth"], 1, hq, d), "bf16"),
                 key=normal(g, (c["depth"], 1, hk, d), "bf16"),
                 value=normal(g, (c["depth"], 1, hk, d), "bf16"))
    retrieval_len = t - c["rejected"]
    return dict(keys=keys, values=values, query=query, steps=steps,
                cos_sin=cos_sin_table(c["budget"], d, c["theta"]), retrieval_len=retrieval_len,
                committed=retrieval_len)


# ---------------------------------------------------------------- KV sink (A9)
# Three requests in reordered canonical slots [3, 1, 2] (a released slot 0),
# prefill written through populate_prefill, one retrieval for the middle
# request, then a draft cycle of 3 steps whose tensors carry 2 graph-padding
# rows after the 3 requests.
CAPTURE = dict(chunk=8, budget=64, depth=3, hk=2, hq=4, d=64, slots=5, max_len=200,
               prompts=(40, 70, 25), padding=2)


def capture_inputs() -> dict:
    c = CAPTURE
    g = rng(1777)
    rows, pad, hk, hq, d = len(c["prompts"]), c["padding"], c["hk"], c["hq"], c["d"]
    total = sum(c["prompts"])
    prefill_pos = np.concatenate([np.arange(n) for n in c["prompts"]]).astype(np.int64)
    steps = []
    for j in range(c["depth"]):
        pos = np.array([n + j for n in c["prompts"]] + [0] * pad, np.int64)
        steps.append(dict(positions=pos, key=normal(g, (rows + pad, hk, d), "bf16"),
                          value=normal(g, (rows + pad, hk, d), "bf16"),
                          query=normal(g, (rows + pad, hq, d), "bf16")))
    n_mid = (c["prompts"][1] + c["chunk"] - 1) // c["chunk"]
    return dict(prefill_positions=prefill_pos, prefill_key=normal(g, (total, hk, d), "bf16"),
                prefill_value=normal(g, (total, hk, d), "bf16"),
                query_ends=np.cumsum(c["prompts"]).astype(np.int64), steps=steps,
                mid_scores=g.random(n_mid, dtype=np.float32),
                cos_sin=round_to(cos_sin_table(c["budget"], d), "bf16"))


# ---------------------------------------------------------- request slots (f)
# Batches passed to set_active_requests one after another on a 6-slot cache:
# a reorder, cancellations, a released id that comes back (a new request), a
# duplicated id, a batch of more distinct requests than slots (exhausted:
# releases and the first assignments happen, then the call raises), the
# batch after it, an empty batch and a fresh start.  Before every call each
# slot in use gets working length 100 + 10 * step + slot and a selection, so
# the fixture shows which slots the call released.
SLOT_COUNT = 6
SLOT_STEPS = (
    ("a", "b", "c"),
    ("c", "a", "b"),
    ("c", "d", "b"),
    ("e", "f", "d", "g"),
    ("a", "e", "e", "h", "i"),
    ("j", "k", "l", "m", "n", "o", "p"),
    ("k", "j"),
    (),
    ("q", "r", "q"),
)
