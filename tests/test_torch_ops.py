"""The torch.library registration of the operator surface (CPU: schemas,
fake implementations, one traced graph; the GPU checks are in
test_gpu_torch_ops.py).  The reference registers its KV sink the same way
(diffspec/vllm_patch.py:130-162) so vLLM's compiled graph holds it as one op."""

from __future__ import annotations

import torch


def _ops(dsb):
    import importlib

    importlib.import_module("vllm-ascend-hust-diffspec_b200.torch_ops")
    return torch.ops.diffspec_b200


def _m(*shape, dt=torch.bfloat16):
    return torch.empty(shape, device="meta", dtype=dt)


def test_schemas_declare_the_in_place_writes(dsb):
    ops = _ops(dsb)
    mutated = {}
    for name in ("paged_chunk_attention_scores", "gather_raw_kv_with_local_rope",
                 "rebuild_compact_kv_from_plan", "rebuild_working_cache", "draft_decode_attention",
                 "capture_raw_kv"):
        schema = getattr(ops, name).default._schema
        mutated[name] = {a.name for a in schema.arguments if a.alias_info and a.alias_info.is_write}
    assert mutated["paged_chunk_attention_scores"] == set()
    assert mutated["gather_raw_kv_with_local_rope"] == set()
    assert mutated["capture_raw_kv"] == set()
    assert mutated["rebuild_compact_kv_from_plan"] == {"working_key", "working_value"}
    assert mutated["draft_decode_attention"] == {"working_key", "working_value", "output"}
    assert mutated["rebuild_working_cache"] == {"working_key", "working_value", "plan",
                                                "history_lens", "working_lens"}
    # keyword names and order of the reference's signatures
    args = [a.name for a in ops.paged_chunk_attention_scores.default._schema.arguments]
    assert args == ["query", "key_cache", "softmax_lse", "block_table", "seq_lens", "chunk_size",
                    "max_seq_len", "scale"]


def test_fake_implementations_give_the_output_shapes(dsb):
    ops = _ops(dsb)
    s = ops.paged_chunk_attention_scores(_m(3, 8, 128), _m(10, 16, 2, 128), None,
                                         _m(3, 5, dt=torch.int32), _m(3, dt=torch.int32), 32, 80, 0.1)
    assert s.shape == (3, 3) and s.dtype == torch.float32
    k, v = ops.gather_raw_kv_with_local_rope(_m(6, 16, 2, 64), _m(6, 16, 2, 64),
                                             _m(2, 3, dt=torch.int32), _m(2, 40, dt=torch.int64),
                                             _m(64, 64), 64, True)
    assert k.shape == v.shape == (2, 40, 2, 64) and k.dtype == torch.bfloat16
    pos = ops.capture_raw_kv(_m(7, dt=torch.int64), _m(7, 256), _m(7, 256), 0)
    assert pos.shape == (7,) and pos.dtype == torch.int64


def test_one_exported_graph_holds_the_path(dsb):
    """Scores, rebuild and attention trace into one graph (no break), in
    order, on fake tensors; nothing runs."""
    ops = _ops(dsb)

    class Cycle(torch.nn.Module):
        def forward(self, q, kc, lse, bt, sl, rk, rv, wk, wv, plan, cs, dq, dk, dv, slots, pos, out):
            s = ops.paged_chunk_attention_scores(q, kc, lse, bt, sl, 32, 80, 0.1)
            ops.rebuild_compact_kv_from_plan(rk, rv, wk, wv, plan, cs, 8, 16, 64, True)
            ops.draft_decode_attention(dq, dk, dv, wk, wv, slots, pos, 0.125, out, 2, 0)
            return s, out

    i32 = torch.int32
    args = (_m(2, 8, 128), _m(10, 16, 2, 128), _m(2, 8, dt=torch.float32), _m(2, 5, dt=i32),
            _m(2, dt=i32), _m(4, 40, 2, 64), _m(4, 40, 2, 64), _m(4, 2, 64, 64), _m(4, 2, 64, 64),
            _m(2, 13, dt=torch.int64), _m(64, 64), _m(2, 8, 64), _m(2, 2, 64), _m(2, 2, 64),
            _m(2, dt=i32), _m(2, dt=i32), _m(2, 8, 64))
    ep = torch.export.export(Cycle(), args)
    called = [str(n.target) for n in ep.graph.nodes if n.op == "call_function"]
    assert called == ["diffspec_b200.paged_chunk_attention_scores.default",
                      "diffspec_b200.rebuild_compact_kv_from_plan.default",
                      "diffspec_b200.draft_decode_attention.default"]


def test_sink_without_a_runtime_returns_the_positions(dsb):
    ops = _ops(dsb)
    import importlib

    t = importlib.import_module("vllm-ascend-hust-diffspec_b200.torch_ops")
    t.set_active_runtime(None)
    pos = torch.arange(5)
    out = ops.capture_raw_kv(pos, torch.zeros(5, 8), torch.zeros(5, 8), 0)
    assert torch.equal(out, pos) and out.data_ptr() != pos.data_ptr()
