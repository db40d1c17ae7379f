"""diffspec_b200 — B200 (sm_100a) DiffSpec draft-context hot path.

A from-scratch CUDA implementation of the draft-context path of the
vllm-ascend-hust-diffspec plugin: chunk-score retrieval over the target's
paged K history, device top-k chunk selection with compact history plans,
the fused gather + local-RoPE working-cache rebuild, and GQA draft decode
attention over the compact cache.  The Python modules keep the reference's
operator surface:

* ``kernels``     — ``paged_chunk_attention_scores``, ``gather_raw_kv_with_local_rope``
* ``compact_kv``  — ``rebuild_compact_kv_from_plan``
* ``selection``   — ``select_context_chunks`` (+ batched/device plan helpers)
* ``attention``   — ``draft_decode_attention``
* ``runtime``     — ``DiffSpecDraftCache`` retrieval hook / rebuild / attention
* ``parallel``    — head-sharded score exchange over NCCL
* ``draft_layer`` — one Eagle3-style draft decoder layer built on the above
* ``torch_ops``   — the same entry points as ``torch.ops.diffspec_b200.*`` custom
  ops (fake implementations, declared in-place writes) for compiled graphs

All compute runs in ``libdiffspec_b200.so`` (C ABI: include/diffspec_b200.h).
The directory name is not a Python identifier; importing it under any name
also registers it (and its submodules) as ``diffspec_b200``.
"""

import sys as _sys

from . import _lib, attention, compact_kv, draft_layer, kernels, parallel, runtime, selection  # noqa: F401
from . import torch_ops  # noqa: F401  (registers torch.ops.diffspec_b200.*)
from .attention import AttentionWorkspace, draft_decode_attention  # noqa: F401
from .compact_kv import rebuild_compact_kv_from_plan  # noqa: F401
from .kernels import (  # noqa: F401
    gather_raw_kv_with_local_rope,
    paged_chunk_attention_scores,
    paged_chunk_head_scores,
)
from .runtime import (  # noqa: F401
    DiffSpecDraftCache,
    DiffSpecSettings,
    chunk_attention_scores,
)
from .selection import DiffSpecSelection, build_history_plan, select_context_chunks, select_rows  # noqa: F401

_sys.modules.setdefault("diffspec_b200", _sys.modules[__name__])
for _name in ("_lib", "attention", "compact_kv", "draft_layer", "kernels", "parallel", "runtime", "selection",
              "torch_ops"):
    _sys.modules.setdefault(f"diffspec_b200.{_name}", _sys.modules[f"{__name__}.{_name}"])



def build_library(force: bool = False):
    """Compile libdiffspec_b200.so for sm_100a (needs nvcc)."""
    import importlib.util
    from pathlib import Path

    spec = importlib.util.spec_from_file_location(
        "_diffspec_b200_build", Path(__file__).resolve().parent / "build.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.build(force=force)
