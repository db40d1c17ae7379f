"""Generate the golden fixtures in this directory by running the REFERENCE.

Runs vllm-ascend-hust-diffspec 0.3.0 from a source checkout (its directory
given by the DIFFSPEC_REFERENCE environment variable) on seeded inputs:

* its PyTorch CPU path (chunk_attention_scores, select_context_chunks,
  DiffSpecDraftCache._history_indices / _history_plan_host /
  _rebuild_working_cache / forward_attention / accept_target_queries /
  populate_prefill / prepare_compact_prefill / capture_raw_kv), including
  BASELINE config 1 as one chain;
* its Triton kernels (paged_chunk_attention_scores,
  rebuild_compact_kv_from_plan, gather_raw_kv_with_local_rope) on the CPU
  under TRITON_INTERPRET=1.

vllm-ascend is not installed, so ref_stubs/ supplies import stand-ins (see
ref_stubs/vllm_ascend/ops/triton/rope.py for the one with math in it).  The
outputs are written as compressed .npz files; bf16 tensors are stored as
uint16 bit patterns (keys ending in "_bf16").

Usage: DIFFSPEC_REFERENCE=<reference checkout> python tests/golden/make_golden.py [names...]
(no names: every fixture; names: e.g. ``config1 capture``).
"""

from __future__ import annotations

import os
import random
import sys
from pathlib import Path
from types import SimpleNamespace

os.environ["TRITON_INTERPRET"] = "1"
HERE = Path(__file__).resolve().parent
if "DIFFSPEC_REFERENCE" not in os.environ:
    raise SystemExit("set DIFFSPEC_REFERENCE to the reference source checkout")
REF = Path(os.environ["DIFFSPEC_REFERENCE"])
sys.path.insert(0, str(HERE / "ref_stubs"))
sys.path.insert(0, str(REF))
sys.path.insert(0, str(HERE.parents[1]))  # repository root: oracle/, tests/golden/recipes.py
sys.path.insert(0, str(HERE))

import numpy as np  # noqa: E402
import torch  # noqa: E402

from diffspec import compact_kv as ref_compact  # noqa: E402
from diffspec import kernels as ref_kernels  # noqa: E402
from diffspec import runtime as ref_rt  # noqa: E402
from vllm.model_executor.layers.rotary_embedding import RotaryEmbedding  # noqa: E402

import recipes as R  # noqa: E402


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def arr(t: torch.Tensor, key: str, out: dict) -> None:
    if t.dtype == torch.bfloat16:
        out[key + "_bf16"] = bits(t)
    elif t.dtype == torch.float16:
        out[key + "_f16"] = t.numpy()
    else:
        out[key] = t.numpy()


_TORCH = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


def T(a: np.ndarray, dtype: str = "f32") -> torch.Tensor:
    """numpy float32 (values exact in `dtype`) -> torch tensor of that dtype."""
    return torch.from_numpy(np.ascontiguousarray(a)).to(_TORCH[dtype])


class Rotary:
    """Rotary object with the attributes DiffSpecDraftCache uses; the CPU
    rotation is vLLM's own RotaryEmbedding.forward_static."""

    def __init__(self, head_dim: int, rotary_dim: int, neox: bool, table: torch.Tensor):
        self.head_size = head_dim
        self.rotary_dim = rotary_dim
        self.is_neox_style = neox
        self.cos_sin_cache = table

    def _match_cos_sin_cache_dtype(self, x):
        return self.cos_sin_cache.to(x.dtype)

    def forward_native(self, positions, query, key=None):
        return RotaryEmbedding.forward_static(
            positions, query, key, self.head_size, self.rotary_dim,
            self._match_cos_sin_cache_dtype(query), self.is_neox_style)


# --------------------------------------------------------------------- scores
def make_scores() -> dict:
    out = {"n": np.array(len(R.SCORE_CASES))}
    for i in range(len(R.SCORE_CASES)):
        inp = R.scores_inputs(i)
        dt = inp["dtype"]
        lse = R.dense_lse(inp)
        query, keys = T(inp["query"], dt), T(inp["key_cache"], dt)
        table = torch.from_numpy(inp["block_table"])
        seq = torch.from_numpy(inp["lengths"])
        triton_scores = ref_kernels.paged_chunk_attention_scores(
            query, keys, torch.from_numpy(lse), table, seq, chunk_size=inp["chunk"],
            max_seq_len=inp["max_len"], scale=inp["scale"])
        p = f"case{i}_"
        out[p + "crc"] = np.array(R.crc(inp["query"], inp["key_cache"], inp["block_table"]))
        out[p + "lse"] = lse
        out[p + "ref_triton_scores"] = triton_scores.numpy()
        bs, hk, d = inp["block_size"], inp["hk"], inp["d"]
        for r, length in enumerate(inp["lengths"]):
            if length == 0:
                continue
            dk = keys[table[r].long()].reshape(-1, hk, d)[:length]
            out[p + f"ref_dense_nolse_row{r}"] = ref_rt.chunk_attention_scores(
                query[r], dk, inp["chunk"], None, inp["scale"]).numpy()
    return out


# --------------------------------------------------------------------- select
def make_select() -> dict:
    cases = R.select_cases()
    out = {"n": np.array(len(cases))}
    for i, (seq_len, c, budget) in enumerate(cases):
        n = (seq_len + c - 1) // c
        scores = R.select_scores(i, n)
        sel = ref_rt.select_context_chunks(torch.from_numpy(scores), seq_len, c, budget)
        p = f"case{i}_"
        out[p + "crc"] = np.array(R.crc(scores))
        out[p + "chunk_indices"] = sel.chunk_indices.numpy()
        out[p + "token_indices"] = sel.token_indices.numpy()
    return out


# --------------------------------------------------------------------- plans
class _IdentityRotary:
    rotary_dim = 0
    is_neox_style = True

    def forward_native(self, positions, query, key=None):
        return query, key


def make_plans() -> dict:
    """The 200-trial plan/indices sweep of tests/test_runtime.py:654-690,
    flattened into one table per chunk size."""
    out = {}
    total = 0
    for chunk in (2, 8, 64):
        rnd = random.Random(17)
        cache = ref_rt.DiffSpecDraftCache(
            ref_rt.DiffSpecSettings(chunk, chunk * 8, 2, 4, 2, 0.7, False),
            max_num_reqs=2, max_model_len=4096, num_kv_heads=1, head_dim=2,
            target_num_layers=2, dtype=torch.float32, device=torch.device("cpu"),
            rotary_embedding=_IdentityRotary(),
        )
        cache.begin_cycle(["a", "b"])
        meta, chunks_flat, plans_flat, idx_flat = [], [], [], []
        for trial in range(200):
            slot = trial % 2
            cache.history_budget = chunk * rnd.randint(1, 7)
            retrieval_end = rnd.randint(1, 3072)
            scores = torch.tensor([rnd.random() for _ in range((retrieval_end + chunk - 1) // chunk)])
            sel = cache.set_chunk_scores(slot, scores, retrieval_end)
            history_end = max(0, retrieval_end + rnd.randint(-4 * chunk, 4 * chunk))
            for kind in ("retrieved", "empty", "none"):
                if kind == "empty":
                    cache._selected_token_indices[slot] = torch.empty(0, dtype=torch.long)
                elif kind == "none":
                    cache._selected_token_indices.pop(slot, None)
                idx = cache._history_indices(slot, history_end).tolist()
                plan = cache._history_plan_host(slot, history_end)
                chunks = sel.chunk_indices.tolist() if kind == "retrieved" else []
                meta.append([cache.history_budget, history_end, slot,
                             {"retrieved": len(chunks), "empty": 0, "none": -1}[kind],
                             len(plan), len(idx)])
                chunks_flat += chunks
                plans_flat += plan
                idx_flat += idx
                total += 1
        p = f"c{chunk}_"
        out[p + "meta"] = np.array(meta, dtype=np.int64)
        out[p + "chunks"] = np.array(chunks_flat, dtype=np.int32)
        out[p + "plans"] = np.array(plans_flat, dtype=np.int64)
        out[p + "indices"] = np.array(idx_flat, dtype=np.int32)
    out["n"] = np.array(total)
    return out


# --------------------------------------------------------------------- rebuild
def make_rebuild() -> dict:
    out = {"n": np.array(len(R.REBUILD_CASES) * len(R.REBUILD_ENDS))}
    k = 0
    for ci in range(len(R.REBUILD_CASES)):
        inp = R.rebuild_inputs(ci)
        heads, dim, rot, neox, slots = (inp[x] for x in ("heads", "dim", "rot", "neox", "slots"))
        table = T(inp["cos_sin"], "bf16")
        cache = ref_rt.DiffSpecDraftCache(
            ref_rt.DiffSpecSettings(R.REBUILD_CHUNK, R.REBUILD_BUDGET, 4, 4, R.REBUILD_DEPTH, 0.7, False),
            max_num_reqs=R.REBUILD_SLOTS, max_model_len=R.REBUILD_LEN, num_kv_heads=heads,
            head_dim=dim, target_num_layers=2, dtype=torch.bfloat16, device=torch.device("cpu"),
            rotary_embedding=Rotary(dim, rot, neox, table),
        )
        cache.raw_key.copy_(T(inp["raw_key"], "bf16"))
        cache.raw_value.copy_(T(inp["raw_value"], "bf16"))
        cache._active_slots = slots
        for end in R.REBUILD_ENDS:
            for slot in slots:
                cache.set_chunk_scores(slot, torch.arange((end + 7) // 8, dtype=torch.float32), end)
            lengths = [end + 1, end + 6]
            plans = [cache._history_plan_host(s, max(0, lengths[r] - 1)) for r, s in enumerate(slots)]
            width = 5 + cache.settings.token_budget // cache.settings.chunk_size
            plan_t = torch.tensor([pl + [0] * (width - len(pl)) for pl in plans], dtype=torch.long)
            max_width = max(pl[1] for pl in plans)
            wk = torch.full(cache.working_key.shape, float("nan")).to(torch.bfloat16)
            wv = wk.clone()
            if max_width:
                ref_compact.rebuild_compact_kv_from_plan(
                    cache.raw_key, cache.raw_value, wk, wv, plan_t, table,
                    chunk_size=R.REBUILD_CHUNK, max_width=max_width, rotary_dim=rot,
                    is_neox_style=neox)
            cache.working_key.fill_(float("nan"))
            cache.working_value.fill_(float("nan"))
            for r in range(2):  # the CPU path cannot rotate an empty history
                if cache._history_indices(slots[r], max(0, lengths[r] - 1)).numel():
                    cache._rebuild_working_cache([r], lengths)
            p = f"case{k}_"
            k += 1
            out[p + "crc"] = np.array(R.crc(inp["raw_key"], inp["raw_value"], inp["cos_sin"]))
            out[p + "meta"] = np.array([ci, end, max_width])
            out[p + "plan"] = plan_t.numpy()
            for r, s in enumerate(slots):
                h = plans[r][1]
                arr(wk[s, :, :h], p + f"row{r}_ref_triton_wk", out)
                # V is a plain copy on both reference paths; keep one flag
                # instead of the tensors.
                out[p + f"row{r}_v_paths_agree"] = np.array(
                    bool(torch.equal(wv[s, :, :h], cache.working_value[s, :, :h])))
                if end >= 62:
                    arr(cache.working_key[s, :, :h], p + f"row{r}_ref_cpu_wk", out)
            untouched = [s for s in range(R.REBUILD_SLOTS) if s not in slots]
            out[p + "untouched_nan"] = np.array(all(torch.isnan(wk[s]).all() for s in untouched))
    return out


# --------------------------------------------------------------------- gather
def make_gather() -> dict:
    out = {"n": np.array(len(R.GATHER_CASES))}
    for i in range(len(R.GATHER_CASES)):
        inp = R.gather_inputs(i)
        k, v = ref_kernels.gather_raw_kv_with_local_rope(
            T(inp["raw_key"], "bf16"), T(inp["raw_value"], "bf16"),
            torch.from_numpy(inp["block_table"]), torch.from_numpy(inp["selected"]),
            T(inp["cos_sin"], "bf16"), rope_dim=inp["rot"], is_neox_style=inp["neox"])
        p = f"case{i}_"
        out[p + "crc"] = np.array(R.crc(inp["raw_key"], inp["raw_value"], inp["selected"]))
        arr(k, p + "ref_key", out)
        arr(v, p + "ref_value", out)
    return out


# --------------------------------------------------------------------- attention
def make_attention() -> dict:
    cases = R.attention_cases()
    out = {"n": np.array(len(cases))}
    for i in range(len(cases)):
        inp = R.attention_inputs(i)
        heads, dim, qheads, budget, slots = cases[i]
        cache = ref_rt.DiffSpecDraftCache(
            ref_rt.DiffSpecSettings(8, budget, 4, 4, 3, 0.7, False),
            max_num_reqs=4, max_model_len=budget, num_kv_heads=heads, head_dim=dim,
            target_num_layers=2, dtype=torch.float32, device=torch.device("cpu"),
            rotary_embedding=_IdentityRotary(),
        )
        cache.working_key.copy_(T(inp["working_key"]))
        cache.working_value.copy_(T(inp["working_value"]))
        p = f"case{i}_"
        out[p + "crc"] = np.array(R.crc(inp["working_key"], inp["working_value"],
                                        *[s[x] for s in inp["steps"] for x in ("query", "key", "value")]))
        for step, st in enumerate(inp["steps"]):
            query = T(st["query"])
            cache._pending_request_indices = list(slots)
            cache._pending_local_positions = [q + step for q in inp["positions"]]
            o = cache.forward_attention(query, T(st["key"]), T(st["value"]), dim ** -0.5,
                                        torch.full_like(query, float("nan")))
            out[p + f"step{step}_ref_out"] = o.numpy()
            out[p + f"step{step}_working_lens"] = np.array(
                [cache._working_lens[s] for s in slots], dtype=np.int32)
    return out


# --------------------------------------------------------------------- hook
def make_hook() -> dict:
    """accept_target_queries with the real (interpreted) Triton scores."""
    out = {"n": np.array(len(R.HOOK_CASES))}
    calls = []
    real = ref_kernels.paged_chunk_attention_scores

    def recorder(query, key_cache, lse, table, lengths, **kw):
        calls.append(lengths.tolist())
        return real(query, key_cache, lse, table, lengths, **kw)

    ref_kernels.paged_chunk_attention_scores = recorder
    try:
        for i in range(len(R.HOOK_CASES)):
            inp = R.hook_inputs(i)
            cache = ref_rt.DiffSpecDraftCache(
                ref_rt.DiffSpecSettings(R.HOOK_CHUNK, R.HOOK_BUDGET, 1, 4, 3, 0.7, False),
                max_num_reqs=2, max_model_len=256, num_kv_heads=R.HOOK_HK, head_dim=R.HOOK_D,
                target_num_layers=2, dtype=torch.float32, device=torch.device("cpu"),
                rotary_embedding=_IdentityRotary(),
            )
            metadata = SimpleNamespace(
                actual_seq_lengths_q=inp["query_ends"].tolist(), seq_lens_list=inp["seq_lens"].tolist(),
                block_tables=torch.from_numpy(inp["block_tables"]), num_prefills=0)
            calls.clear()
            cache.begin_target_forward(["a", "b"])
            cache.capture_target_attention(T(inp["query"], "bf16"), torch.from_numpy(inp["lse"]),
                                           T(inp["key_cache"], "bf16"), metadata, R.HOOK_D ** -0.5)
            cache.accept_target_queries(torch.from_numpy(inp["counts"]), is_prefill=False)
            p = f"case{i}_"
            out[p + "crc"] = np.array(R.crc(inp["query"], inp["lse"], inp["key_cache"]))
            out[p + "history_budget"] = np.array(cache.history_budget)
            out[p + "ref_lengths"] = np.array(calls[0] if calls else [], dtype=np.int32)
            for slot in range(2):
                sel = cache._selected_token_indices.get(slot)
                out[p + f"ref_selected_slot{slot}"] = (
                    np.array([-2]) if sel is None else sel.numpy().astype(np.int64))
            status = cache.retrieval_status()
            out[p + "ref_status"] = np.array([status["retrieval_count"],
                                              status["retrieval_skipped_no_committed_tokens"]])
    finally:
        ref_kernels.paged_chunk_attention_scores = real
    return out


# --------------------------------------------------------------------- config 1
def make_config1() -> dict:
    """BASELINE config 1 as one chain of the reference's CPU path:
    chunk_attention_scores (LSE computed) -> set_chunk_scores /
    select_context_chunks -> _rebuild_working_cache -> forward_attention for
    the K draft steps, in fp32."""
    c, inp = R.CONFIG1, R.config1_inputs()
    d, hq, hk = c["d"], c["hq"], c["hk"]
    scale = d ** -0.5
    L = inp["retrieval_len"]
    scores = ref_rt.chunk_attention_scores(T(inp["query"]), T(inp["keys"][:L]), c["chunk"], None, scale)
    cache = ref_rt.DiffSpecDraftCache(
        ref_rt.DiffSpecSettings(c["chunk"], c["budget"], 1, 4, c["depth"], 0.7, False),
        max_num_reqs=1, max_model_len=c["tokens"], num_kv_heads=hk, head_dim=d,
        target_num_layers=2, dtype=torch.float32, device=torch.device("cpu"),
        rotary_embedding=Rotary(d, d, True, T(inp["cos_sin"])),
    )
    cache.raw_key[0].copy_(T(inp["keys"]))
    cache.raw_value[0].copy_(T(inp["values"]))
    cache.begin_cycle(["r"])
    sel = cache.set_chunk_scores(0, scores, L)
    plan = cache._history_plan_host(0, inp["committed"] - 1)
    local = cache._rebuild_working_cache([0], [inp["committed"]])
    out = {"n": np.array(1), "crc": np.array(R.crc(inp["keys"], inp["values"], inp["query"])),
           "history_budget": np.array(cache.history_budget), "scores": scores.numpy(),
           "chunk_indices": sel.chunk_indices.numpy(), "token_indices": sel.token_indices.numpy(),
           "plan": np.array(plan, np.int64), "local_positions": np.array(local, np.int64),
           "working_key": cache.working_key[0, :, : local[0]].numpy().copy()}
    st = inp["steps"]
    for j in range(c["depth"]):
        cache._pending_request_indices = [0]
        cache._pending_local_positions = [local[0] + j]
        query = T(st["query"][j])
        o = cache.forward_attention(query, T(st["key"][j]), T(st["value"][j]), scale,
                                    torch.full_like(query, float("nan")))
        out[f"step{j}_out"] = o.numpy().copy()
    out["working_lens"] = np.array([cache._working_lens[0]], np.int64)
    return out


# --------------------------------------------------------------------- KV sink
def make_capture() -> dict:
    """populate_prefill -> set_chunk_scores -> prepare_compact_prefill ->
    (capture_raw_kv -> forward_attention) per draft step, with graph padding
    rows, on the reference's CPU path (fp32 caches: its CPU attention loop
    needs them; the inputs are exact in bf16); the forward context's
    attention metadata is supplied directly."""
    c, inp = R.CAPTURE, R.capture_inputs()
    d, hk = c["d"], c["hk"]
    cache = ref_rt.DiffSpecDraftCache(
        ref_rt.DiffSpecSettings(c["chunk"], c["budget"], 1, 4, c["depth"], 0.7, False),
        max_num_reqs=c["slots"], max_model_len=c["max_len"], num_kv_heads=hk, head_dim=d,
        target_num_layers=2, dtype=torch.float32, device=torch.device("cpu"),
        rotary_embedding=Rotary(d, d, True, T(inp["cos_sin"])),
    )
    cache.raw_key.zero_()
    cache.raw_value.zero_()
    ids = ["c", "a", "b"]
    cache.set_active_requests(["x", "a", "b", "c"])
    cache.set_active_requests(ids)  # slots [3, 1, 2]: "x" released slot 0
    prompts = list(c["prompts"])
    prefill_meta = SimpleNamespace(actual_seq_lengths_q=inp["query_ends"].tolist())
    cache.populate_prefill(torch.from_numpy(inp["prefill_positions"]), T(inp["prefill_key"]),
                           T(inp["prefill_value"]), prefill_meta)
    sel = cache.set_chunk_scores(cache._active_slots[1], torch.from_numpy(inp["mid_scores"]), prompts[1])
    out = {"n": np.array(1), "active_slots": np.array(cache._active_slots, np.int64),
           "crc": np.array(R.crc(inp["prefill_key"], inp["prefill_value"], inp["mid_scores"])),
           "mid_chunks": sel.chunk_indices.numpy()}
    cache.begin_cycle(ids)
    committed = [n + 1 for n in prompts]  # the root at position n is the cycle's first token
    meta = SimpleNamespace(seq_lens_list=committed, actual_seq_lengths_q=[1, 2, 3])
    cache._first_attention_metadata = lambda: meta
    cache.prepare_compact_prefill(meta, len(ids), committed_seq_lens=committed)
    for j, st in enumerate(inp["steps"]):
        pos = cache.capture_raw_kv(0, torch.from_numpy(st["positions"]), T(st["key"]),
                                   T(st["value"]))
        query = T(st["query"])
        o = cache.forward_attention(query, T(st["key"]), T(st["value"]), d ** -0.5,
                                    torch.full_like(query, float("nan")))
        out[f"step{j}_local_positions"] = pos.numpy().copy()
        arr(o, f"step{j}_out", out)
    cache.end_cycle()
    arr(cache.raw_key, "raw_key", out)
    arr(cache.raw_value, "raw_value", out)
    arr(cache.working_key, "working_key", out)
    arr(cache.working_value, "working_value", out)
    out["working_lens"] = np.array([int(cache._working_lens[s]) for s in range(c["slots"])], np.int64)
    return out


# ------------------------------------------------------------- request slots
def make_slots() -> dict:
    """set_active_requests over recipes.SLOT_STEPS on the reference's cache:
    before each call every slot in use gets a working length and a
    selection; after it, the active slots (unchanged when the call raised),
    whether it raised, the working lengths and which slots keep a
    selection."""
    cache = ref_rt.DiffSpecDraftCache(
        ref_rt.DiffSpecSettings(8, 64, 1, 4, 3, 0.7, False), max_num_reqs=R.SLOT_COUNT,
        max_model_len=32, num_kv_heads=1, head_dim=64, target_num_layers=2,
        dtype=torch.float32, device=torch.device("cpu"),
        rotary_embedding=Rotary(64, 64, True, torch.zeros((64, 64))),
    )
    out = {"n": np.array(len(R.SLOT_STEPS))}
    for i, batch in enumerate(R.SLOT_STEPS):
        for slot in cache._request_slots.values():
            cache._working_lens[slot] = 100 + 10 * i + slot
            cache._selected_token_indices[slot] = torch.zeros(1, dtype=torch.long)
        raised = 0
        try:
            cache.set_active_requests(list(batch))
        except RuntimeError as error:
            assert "exhausted" in str(error)
            raised = 1
        out[f"active{i}"] = np.array(cache._active_slots, np.int64)
        out[f"raised{i}"] = np.array(raised)
        out[f"working_lens{i}"] = np.array(cache._working_lens, np.int64)
        sel = np.zeros(R.SLOT_COUNT, np.int64)
        sel[list(cache._selected_token_indices)] = 1
        out[f"selected{i}"] = sel
    return out


FIXTURES = (("scores", "make_scores"), ("select", "make_select"), ("plans", "make_plans"),
            ("rebuild", "make_rebuild"), ("gather", "make_gather"), ("attention", "make_attention"),
            ("hook", "make_hook"), ("config1", "make_config1"), ("capture", "make_capture"),
            ("slots", "make_slots"))


def main() -> None:
    """Writes every fixture, or only those named on the command line."""
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    wanted = set(sys.argv[1:])
    for name, fn_name in FIXTURES:
        if wanted and name not in wanted:
            continue
        data = globals()[fn_name]()
        path = HERE / f"{name}.npz"
        np.savez_compressed(path, **data)
        print(f"{path.name}: {int(data['n'])} cases, {path.stat().st_size / 1024:.0f} KiB")


if __name__ == "__main__":
    main()
