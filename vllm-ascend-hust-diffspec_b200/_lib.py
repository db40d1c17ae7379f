"""ctypes binding of libdiffspec_b200.so (the C ABI in include/diffspec_b200.h).

The shared library is the only compute path of this package: there is no
Triton, no PyTorch re-implementation and no CPU fallback.  Loading fails
loudly when the library is missing; callers on a machine without a GPU can
still load it (it only needs the CUDA driver at call time) to inspect the ABI.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libdiffspec_b200.so"

DSB_OK = 0
DSB_ERR_INVALID = 1
DSB_ERR_UNSUPPORTED = 2
DSB_ERR_CUDA = 3

DSB_BF16 = 0
DSB_F16 = 1
DSB_F32 = 2

DSB_FLAG_SLOT = 1
DSB_FLAG_POSITION = 2

FLAG_NAMES = {
    1: "slot out of range",
    2: "token position out of range",
    4: "block-table entry out of range",
    8: "malformed plan row",
    16: "selection exceeds per-slot capacity",
    32: "bounded wait for an asynchronous copy ran out",
}

_DTYPE_CODES = {
    torch.bfloat16: DSB_BF16,
    torch.float16: DSB_F16,
    torch.float32: DSB_F32,
}

_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64
_F32 = ctypes.c_float

# name -> (restype, argtypes), in header order.
_SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "dsb_last_error": (ctypes.c_char_p, []),
    "dsb_abi_version": (ctypes.c_int, []),
    "dsb_paged_chunk_head_scores": (
        ctypes.c_int,
        [_P, _P, _P, _I32, _P, _P, _I64, _I64, _P, _I32, _I32, _I32, _I32, _I32, _I64, _I32, _I32,
         _F32, _I32, _P, _P, _P],
    ),
    "dsb_paged_chunk_stats": (
        ctypes.c_int,
        [_P, _P, _I32, _P, _P, _I64, _I64, _P, _I32, _I32, _I32, _I32, _I32, _I64, _I32, _I32, _F32,
         _I32, _P, _P, _P, _P],
    ),
    "dsb_chunk_stats_to_head_scores": (
        ctypes.c_int,
        [_P, _P, _P, _I32, _I32, _I32, _I32, _I32, _P, _P, _P],
    ),
    "dsb_finalize_chunk_scores": (
        ctypes.c_int,
        [_P, _I64, _I64, _I32, _P, _I32, _I32, _I32, _I32, _P, _P],
    ),
    "dsb_select_context_chunks": (
        ctypes.c_int,
        [_P, _I64, _I64, _I32, _I32, _I64, _I32, _P, _P, _I32, _I32, _I32, _I32, _I32, _P, _I32,
         _P, _I32, _P, _P, _P, _P, _P],
    ),
    "dsb_build_history_plan": (
        ctypes.c_int,
        [_P, _P, _I32, _P, _I32, _P, _I32, _I32, _I32, _I32, _I32, _P, _P, _P, _P, _P],
    ),
    "dsb_rebuild_compact_kv_from_plan": (
        ctypes.c_int,
        [_P, _P, _P, _P, _P, _I32, _I32, _P, _I32, _I64, _I64, _I32, _I64, _I32, _I32, _I32,
         _I32, _I32, _I32, _I32, _I32, _P, _P],
    ),
    "dsb_rebuild_working_cache": (
        ctypes.c_int,
        [_P, _P, _P, _P, _P, _P, _I32, _P, _I32, _P, _I32, _I32, _I32, _I32, _I32, _P, _P, _P, _P,
         _I32, _I64, _I64, _I64, _I32, _I32, _I32, _I32, _I32, _I32, _P, _P],
    ),
    "dsb_kv_projection_write_raw": (
        ctypes.c_int,
        [_P, _I32, _I32, _P, _I32, _I32, _P, _P, _P, _P, _I32, _I64, _I32, _P, _P, _P],
    ),
    "dsb_paged_decode_scratch_floats": (_I64, [_I32, _I32, _I32, _I32]),
    "dsb_paged_decode_attention_lse": (
        ctypes.c_int,
        [_P, _I32, _I32, _I32, _I32, _P, _P, _I64, _I32, _P, _I64, _I64, _I64, _P, _P, _I32, _F32,
         _I32, _I32, _P, _P, _P, _I64, _P, _P],
    ),
    "dsb_qkv_projection_write_raw": (
        ctypes.c_int,
        [_P, _I32, _I32, _P, _I32, _I32, _I32, _P, _P, _P, _P, _I32, _I64, _I32, _P, _P, _I32,
         _P, _P],
    ),
    "dsb_pack_linear_weight": (ctypes.c_int, [_P, _I64, _I32, _I32, _P, _P]),
    "dsb_draft_linear": (
        ctypes.c_int,
        [_P, _I32, _I32, _P, _I32, _I32, _P, _I64, _P, _I64, _I32, _I32, _P, _P],
    ),
    "dsb_add_rms_norm": (
        ctypes.c_int, [_P, _I64, _P, _I64, _P, _P, _I64, _P, _I64, _I32, _I32, _F32, _I32, _P]),
    "dsb_rms_norm": (ctypes.c_int, [_P, _I64, _P, _P, _I64, _I32, _I32, _F32, _I32, _P]),
    "dsb_rope_qk": (
        ctypes.c_int,
        [_P, _I64, _I32, _P, _I64, _P, _P, _I64, _P, _I32, _I32, _P, _I32, _I32, _P, _I64, _I32,
         _I32, _I32, _P, _P],
    ),
    "dsb_silu_mul": (ctypes.c_int, [_P, _I64, _P, _I64, _I32, _I32, _I32, _P]),
    "dsb_gather_raw_kv_with_local_rope": (
        ctypes.c_int,
        [_P, _P, _I64, _I32, _I32, _I32, _P, _I64, _I64, _P, _I32, _I32, _P, _I32, _I64, _I64,
         _I32, _I32, _I32, _P, _P, _P, _P],
    ),
    "dsb_draft_decode_attention": (
        ctypes.c_int,
        [_P, _P, _P, _P, _P, _P, _P, _I32, _I32, _I32, _I32, _I32, _I32, _I32, _I32, _F32, _I32, _P,
         _P, _I64, _P, _I32, _P, _P],
    ),
    "dsb_draft_decode_attention_static": (
        ctypes.c_int,
        [_P, _P, _P, _P, _P, _P, _P, _I32, _I32, _I32, _I32, _I32, _I32, _I32, _I32, _F32, _I32,
         _P, _I32, _P, _P],
    ),
    "dsb_draft_attention_default_splits": (_I32, [_I32, _I32, _I32, _I32]),
    "dsb_draft_attention_scratch_floats": (_I64, [_I32, _I32, _I32, _I32, _I32]),
    "dsb_prepare_retrieval_rows": (
        ctypes.c_int,
        [_P, _P, _P, _I32, _P, _I32, _P, _P, _P, _P, _P],
    ),
    "dsb_write_raw_kv": (
        ctypes.c_int,
        [_P, _P, _P, _P, _P, _P, _I32, _I32, _I64, _I32, _I32, _I32, _P, _P],
    ),
    "dsb_capture_raw_kv": (
        ctypes.c_int,
        [_P, _P, _I64, _P, _P, _P, _P, _I32, _I32, _I32, _I32, _I64, _I32, _I32, _I32, _P, _I32,
         _I32, _P, _P, _P, _P],
    ),
    "dsb_peer_buffer_bytes": (_I64, [_I32, _I32, _I32]),
    "dsb_peer_buffer_create": (ctypes.c_int, [_I32, _I32, _I32, ctypes.POINTER(ctypes.c_void_p)]),
    "dsb_peer_buffer_destroy": (ctypes.c_int, [_P]),
    "dsb_ipc_handle": (ctypes.c_int, [_P, _P]),
    "dsb_ipc_open": (ctypes.c_int, [_P, ctypes.POINTER(ctypes.c_void_p)]),
    "dsb_ipc_close": (ctypes.c_int, [_P]),
    "dsb_draft_linear_peer": (
        ctypes.c_int, [_P, _I32, _I32, _P, _I32, _P, _I32, _I32, _I32, _P, _I32, _I32, _P, _P]),
    "dsb_peer_all_gather_send": (ctypes.c_int, [_P, _I64, _P, _I32, _I32, _I64, _P, _P]),
    "dsb_peer_all_gather_recv": (ctypes.c_int, [_P, _I32, _I64, _I64, _P, _P, _P]),
    "dsb_peer_add_rms_norm": (
        ctypes.c_int,
        [_P, _I32, _I32, _P, _I64, _P, _P, _I64, _P, _I64, _I32, _I32, _F32, _I32, _P, _P]),
    "dsb_assign_request_slots": (
        ctypes.c_int, [_P, _I32, _P, _I32, _P, _P, _P, _P, _P, _P],
    ),
    "dsb_rows_to_slots": (ctypes.c_int, [_P, _I32, _P, _I32, _P, _P, _P]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load the shared library once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH.name} is missing: build it with "
                    "`python vllm-ascend-hust-diffspec_b200/build.py` (needs nvcc); "
                    "the DiffSpec B200 ops have no fallback implementation"
                )
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (restype, argtypes) in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _lib = lib
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPE_CODES[dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {dtype}") from None


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_ptr(device: torch.device) -> int:
    """The current CUDA stream of `device` as a raw pointer (the cheap C-level
    query when this PyTorch has it)."""
    if _raw_stream is not None:
        idx = device.index if device.index is not None else torch.cuda.current_device()
        return _raw_stream(idx)
    return torch.cuda.current_stream(device).cuda_stream


def check(status: int, what: str) -> None:
    if status == DSB_OK:
        return
    msg = load().dsb_last_error().decode(errors="replace")
    if status == DSB_ERR_INVALID:
        raise ValueError(f"{what}: {msg}")
    raise RuntimeError(f"{what}: {msg} (status {status})")


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)


_error_flags: dict[int, torch.Tensor] = {}
_sm_counts: dict[int, int] = {}


def error_flag(device: torch.device) -> torch.Tensor:
    """Per-device int32 word the kernels OR bad-index bits into."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    flag = _error_flags.get(idx)
    if flag is None:
        flag = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _error_flags[idx] = flag
    return flag


def read_and_clear_error_flag(device: torch.device) -> int:
    flag = error_flag(device)
    value = int(flag.item())
    flag.zero_()
    return value


def describe_flag(value: int) -> str:
    return ", ".join(name for bit, name in FLAG_NAMES.items() if value & bit) or "none"


def sm_count(device: torch.device) -> int:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    n = _sm_counts.get(idx)
    if n is None:
        n = torch.cuda.get_device_properties(idx).multi_processor_count
        _sm_counts[idx] = n
    return n


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    """All tensors on one CUDA device, 16-byte aligned; returns the device."""
    device = None
    for t in tensors:
        if t is None:
            continue
        if t.device.type != "cuda":
            raise ValueError("DiffSpec B200 ops need CUDA tensors (there is no CPU path)")
        if device is None:
            device = t.device
        elif t.device != device:
            raise ValueError("all tensors must share one CUDA device")
    if device is None:
        raise ValueError("no tensor arguments")
    return device
