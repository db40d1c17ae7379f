"""The C ABI: the library loads without a GPU, exports exactly what
include/diffspec_b200.h declares, and rejects bad arguments before launching."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

from conftest import ROOT


def _declared() -> set[str]:
    text = (ROOT / "include" / "diffspec_b200.h").read_text()
    return set(re.findall(r"\b(dsb_\w+)\s*\(", text))


def test_header_symbols_are_exported_and_bound(dsb):
    lib = dsb._lib.load()
    declared = _declared()
    assert declared, "no declarations found"
    for name in declared:
        assert hasattr(lib, name), name
    assert declared == set(dsb._lib.exported_symbols())
    assert lib.dsb_abi_version() == 2


def test_library_is_the_in_tree_build(dsb):
    maps = Path("/proc/self/maps").read_text()
    assert str(dsb._lib.LIB_PATH) in maps


def test_invalid_arguments_fail_before_any_launch(dsb):
    lib = dsb._lib.load()
    # budget not a multiple of the chunk size
    def select(budget=64, window=0, per_group=0, parts=1):
        return lib.dsb_select_context_chunks(ctypes.c_void_p(8), 0, 0, parts, per_group, 0, 0,
                                             ctypes.c_void_p(8), None, 1, 10, 16, budget, window,
                                             None, 0, None, 0, None, None, None, None, None)

    assert select(budget=50) == dsb._lib.DSB_ERR_INVALID
    assert b"chunk-size multiple" in lib.dsb_last_error()
    # rolling recent window: a chunk multiple within [chunk, budget]
    for window in (8, 24, 80):
        assert select(window=window) == dsb._lib.DSB_ERR_INVALID
        assert b"recent_window" in lib.dsb_last_error()
    # grouped parts must tile the part count
    assert select(parts=4, per_group=3) == dsb._lib.DSB_ERR_INVALID
    assert b"parts_per_group" in lib.dsb_last_error()
    fake = ctypes.c_void_p(256)
    assert lib.dsb_build_history_plan(fake, fake, 1, fake, 4, fake, 4, 16, 64, 24, 9, fake, None,
                                      None, None, None) == dsb._lib.DSB_ERR_INVALID
    assert b"recent_window" in lib.dsb_last_error()
    # plan width must be 5 + W / C
    st = lib.dsb_rebuild_compact_kv_from_plan(None, None, None, None, None, 1, 7, None, 0, 0, 0, 1,
                                              8, 1, 64, 64, 8, 8, 64, 1, 0, None, None)
    assert st == dsb._lib.DSB_ERR_INVALID and b"plan width" in lib.dsb_last_error()
    # attention: unsupported head_dim is reported, not launched
    st = lib.dsb_draft_decode_attention(None, None, None, None, None, None, None, 0, 1, 1, 1, 8, 1,
                                        96, 64, 0.1, 0, None, None, 0, None, 1, None, None)
    assert st == dsb._lib.DSB_ERR_UNSUPPORTED
    # empty work is a no-op success
    assert lib.dsb_write_raw_kv(None, None, None, None, None, None, 0, 1, 1, 1, 8, 0, None, None) == 0
    # request slots: table size in [1, 4096], requests in [0, 4096], a table
    assert lib.dsb_assign_request_slots(fake, 0, fake, 1, fake, None, None, None, None,
                                        None) == dsb._lib.DSB_ERR_INVALID
    assert lib.dsb_assign_request_slots(fake, 4097, fake, 1, fake, None, None, None, None,
                                        None) == dsb._lib.DSB_ERR_INVALID
    assert lib.dsb_assign_request_slots(fake, 8, fake, 5000, fake, None, None, None, None,
                                        None) == dsb._lib.DSB_ERR_INVALID
    assert lib.dsb_assign_request_slots(None, 8, fake, 1, fake, None, None, None, None,
                                        None) == dsb._lib.DSB_ERR_INVALID
    assert lib.dsb_rows_to_slots(fake, 1, fake, -1, fake, None, None) == dsb._lib.DSB_ERR_INVALID
    assert lib.dsb_rows_to_slots(None, 1, None, 0, None, None, None) == 0


def test_split_and_scratch_helpers(dsb):
    lib = dsb._lib.load()
    splits = lib.dsb_draft_attention_default_splits(16, 4, 2048, 148)
    assert 1 <= splits <= 64
    assert lib.dsb_draft_attention_scratch_floats(16, 32, 4, 128, splits) == 16 * 4 * splits * 8 * 130
    assert lib.dsb_draft_attention_scratch_floats(2, 32, 2, 128, 3) == 2 * 2 * 3 * 16 * 130


def test_draft_layer_entry_points_reject_bad_arguments(dsb):
    """The draft-layer entry points validate on the host: no device pointer
    is dereferenced (fake non-null addresses) and nothing is launched."""
    lib = dsb._lib.load()
    P, L = dsb._lib, lib
    fake = ctypes.c_void_p(256)
    # linear: unknown epilogue, K not a multiple of 64, rows not a multiple of 128,
    # output stride shorter than a row, residual missing
    assert L.dsb_draft_linear(fake, 16, 128, fake, 128, 7, None, 0, fake, 128, 0, 0, None, None) \
        == P.DSB_ERR_INVALID
    assert b"epilogue" in L.dsb_last_error()
    assert L.dsb_draft_linear(fake, 16, 100, fake, 128, 0, None, 0, fake, 128, 0, 0, None, None) \
        == P.DSB_ERR_UNSUPPORTED
    assert L.dsb_draft_linear(fake, 16, 128, fake, 96, 0, None, 0, fake, 96, 0, 0, None, None) \
        == P.DSB_ERR_UNSUPPORTED
    assert L.dsb_draft_linear(fake, 16, 128, fake, 256, 2, None, 0, fake, 100, 0, 0, None, None) \
        == P.DSB_ERR_INVALID  # SwiGLU output has 128 columns
    assert L.dsb_draft_linear(fake, 16, 128, fake, 128, 1, None, 0, fake, 128, 0, 0, None, None) \
        == P.DSB_ERR_INVALID
    assert b"residual" in L.dsb_last_error()
    assert L.dsb_draft_linear(fake, 16, 128, fake, 128, 0, None, 0, fake, 128, 5, 0, None, None) \
        == P.DSB_ERR_INVALID  # fp32 is not a tensor-core operand type here
    assert L.dsb_draft_linear(fake, 0, 128, fake, 128, 0, None, 0, fake, 128, 0, 0, None, None) \
        == P.DSB_OK  # no tokens: nothing to do
    # qkv projection: q features not a multiple of 128, missing q output
    args = [fake, 16, 256, fake, 100, 1, 128, fake, fake, fake, fake, 4, 64, 0, fake, fake, 0, None,
            None]
    assert L.dsb_qkv_projection_write_raw(*args) == P.DSB_ERR_UNSUPPORTED
    args[4], args[14] = 128, None
    assert L.dsb_qkv_projection_write_raw(*args) == P.DSB_ERR_INVALID
    # weight packing: rows not a multiple of 128, cols not of 64, aliased buffers
    assert L.dsb_pack_linear_weight(fake, 100, 64, 0, ctypes.c_void_p(512), None) == P.DSB_ERR_UNSUPPORTED
    assert L.dsb_pack_linear_weight(fake, 128, 96, 0, ctypes.c_void_p(512), None) == P.DSB_ERR_UNSUPPORTED
    assert L.dsb_pack_linear_weight(fake, 128, 64, 0, fake, None) == P.DSB_ERR_INVALID
    # elementwise stages
    assert L.dsb_rms_norm(fake, 12, fake, fake, 12, 2, 12, 1e-6, 0, None) == P.DSB_ERR_UNSUPPORTED
    assert L.dsb_rms_norm(fake, 16, fake, fake, 16, 2, 16, -1.0, 0, None) == P.DSB_ERR_INVALID
    assert L.dsb_silu_mul(fake, 8, fake, 8, 2, 8, 0, None) == P.DSB_ERR_UNSUPPORTED  # row < 2 * inter
    assert L.dsb_rope_qk(fake, 256, 2, fake, 200, fake, None, 0, None, 2, 128, fake, 0, 3, fake, 128,
                         64, 0, 0, None, None) == P.DSB_ERR_INVALID  # key row < 2 heads * 128
    assert L.dsb_rope_qk(fake, 256, 2, fake, 256, fake, None, 0, None, 2, 127, fake, 0, 3, fake, 128,
                         64, 0, 0, None, None) == P.DSB_ERR_INVALID  # odd head_dim


def test_target_attention_rejects_bad_arguments(dsb):
    lib = dsb._lib.load()
    P = dsb._lib
    fake = ctypes.c_void_p(256)
    ok = [fake, 4, 32, 4, 128, fake, fake, 100, 16, fake, 8, 4, 8, fake, None, 128, 0.088, 0, 512,
          fake, fake, fake, 10 ** 6, None, None]

    def call(**over):
        a = list(ok)
        for i, v in over.items():
            a[int(i[1:])] = v
        return lib.dsb_paged_decode_attention_lse(*a)

    assert call(a4=64) == P.DSB_ERR_UNSUPPORTED          # head_dim 64
    assert call(a2=30) == P.DSB_ERR_INVALID              # 30 query heads over 4 kv heads
    assert call(a16=0.0) == P.DSB_ERR_INVALID            # scale
    assert call(a22=10) == P.DSB_ERR_INVALID             # scratch too small
    assert b"scratch" in lib.dsb_last_error()
    assert call(a10=4) == P.DSB_ERR_INVALID              # table stride shorter than its columns
    assert call(a17=2) == P.DSB_ERR_INVALID              # fp32 caches
    assert call(a1=0) == P.DSB_OK                        # no rows
    assert lib.dsb_paged_decode_scratch_floats(4, 32, 1000, 512) == 4 * 32 * 2 * 130
    # default split length: 512 tokens below 16384, 1024 from there on
    assert lib.dsb_paged_decode_scratch_floats(4, 32, 1000, 0) == 4 * 32 * 2 * 130
    assert lib.dsb_paged_decode_scratch_floats(4, 32, 40960, 0) == 4 * 32 * 40 * 130


def test_peer_exchange_entry_points_reject_bad_arguments(dsb):
    """The fused all-reduce / all-gather entry points and the exchange buffer
    helpers validate on the host, before any CUDA call."""
    lib = dsb._lib.load()
    inv = dsb._lib.DSB_ERR_INVALID
    fake = ctypes.c_void_p(256)
    # buffer size: 2 parities x world x tokens x features words of 8 bytes, then
    # the 128-byte-aligned sync words
    data = 2 * 2 * 16 * 2048 * 8
    assert lib.dsb_peer_buffer_bytes(2, 16, 2048) == (data + 127) // 128 * 128 + 128
    assert lib.dsb_peer_buffer_bytes(0, 16, 2048) == -1
    assert lib.dsb_peer_buffer_bytes(9, 16, 2048) == -1
    base = ctypes.c_void_p()
    assert lib.dsb_peer_buffer_create(9, 16, 2048, ctypes.byref(base)) == inv
    assert lib.dsb_peer_buffer_create(2, 16, 2047, ctypes.byref(base)) == inv
    assert lib.dsb_peer_buffer_destroy(None) == 0 and lib.dsb_ipc_close(None) == 0
    assert lib.dsb_ipc_handle(None, fake) == inv and lib.dsb_ipc_open(None, ctypes.byref(base)) == inv
    # linear + all-reduce: rank within world, tokens within the buffer
    assert lib.dsb_draft_linear_peer(fake, 16, 64, fake, 128, fake, 2, 2, 16, fake, 0, 0, None,
                                     None) == inv
    assert lib.dsb_draft_linear_peer(fake, 17, 64, fake, 128, fake, 2, 0, 16, fake, 0, 0, None,
                                     None) == inv
    assert lib.dsb_peer_add_rms_norm(fake, 2, 16, fake, 128, None, fake, 128, None, 0, 17, 128,
                                     1e-6, 0, None, None) == inv
    # all-gather: counts are multiples of 8 within the buffer's row
    assert lib.dsb_peer_all_gather_send(fake, 12, fake, 2, 0, 64, fake, None) == inv
    assert lib.dsb_peer_all_gather_send(fake, 72, fake, 2, 0, 64, fake, None) == inv
    assert lib.dsb_peer_all_gather_recv(fake, 2, 12, 64, fake, None, None) == inv
    assert lib.dsb_peer_all_gather_send(fake, 0, fake, 2, 0, 64, fake, None) == 0
