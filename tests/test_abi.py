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
    assert lib.dsb_abi_version() == 1


def test_library_is_the_in_tree_build(dsb):
    maps = Path("/proc/self/maps").read_text()
    assert str(dsb._lib.LIB_PATH) in maps


def test_invalid_arguments_fail_before_any_launch(dsb):
    lib = dsb._lib.load()
    # budget not a multiple of the chunk size
    st = lib.dsb_select_context_chunks(ctypes.c_void_p(8), 0, 0, 1, 0, ctypes.c_void_p(8), None, 1, 10, 16, 50,
                                       None, 0, None, 0, None, None, None, None, None)
    assert st == dsb._lib.DSB_ERR_INVALID
    assert b"chunk-size multiple" in lib.dsb_last_error()
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


def test_split_and_scratch_helpers(dsb):
    lib = dsb._lib.load()
    splits = lib.dsb_draft_attention_default_splits(16, 4, 2048, 148)
    assert 1 <= splits <= 64
    assert lib.dsb_draft_attention_scratch_floats(16, 32, 4, 128, splits) == 16 * 4 * splits * 8 * 130
    assert lib.dsb_draft_attention_scratch_floats(2, 32, 2, 128, 3) == 2 * 2 * 3 * 16 * 130
