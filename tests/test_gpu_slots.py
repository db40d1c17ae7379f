"""Request slots on the device: DiffSpecDraftCache.set_active_requests runs
dsb_assign_request_slots over a device slot table.  Checked against the
reference's own set_active_requests run (tests/golden/slots.npz, made by
tests/golden/make_golden.py; diffspec/runtime.py:755-778) and against the
oracle's restatement over long random batch sequences: the slots of every
batch, which call raises (exhaustion), and the per-slot state a release
resets (working length 0, no selection)."""

from __future__ import annotations

import ctypes
import random

import numpy as np
import pytest
import torch

import recipes as R
from conftest import golden
from oracle import diffspec_oracle as O

pytestmark = pytest.mark.gpu


def _cache(dsb, cuda, slots):
    settings = dsb.runtime.DiffSpecSettings(8, 64, 1, 4, 3, 0.7, False)
    return dsb.runtime.DiffSpecDraftCache(
        settings, max_num_reqs=slots, max_model_len=32, num_kv_heads=1, head_dim=64,
        target_num_layers=2, dtype=torch.bfloat16, device=cuda,
        cos_sin_cache=torch.zeros((64, 64), device=cuda))


def _mark_in_use(cache, step):
    """Every slot in use gets working length 100 + 10 * step + slot and a
    selection, as the fixture's run does before each call."""
    used = cache._slot_keys >= 0
    idx = torch.arange(cache.max_num_reqs, device=cache.device, dtype=torch.int32)
    cache.working_lens.copy_(torch.where(used, 100 + 10 * step + idx, cache.working_lens))
    cache.sel_count.copy_(torch.where(used, torch.ones_like(cache.sel_count), cache.sel_count))


def _call(cache, batch):
    try:
        cache.set_active_requests(list(batch))
    except RuntimeError as error:
        assert "exhausted" in str(error)
        return 1
    return 0


def _state(cache):
    return (cache.active_slots(), cache.working_lens.cpu().tolist(),
            torch.nonzero(cache.sel_count >= 0).flatten().cpu().tolist())


def test_slots_match_reference_run(dsb, cuda):
    d = golden("slots")
    cache = _cache(dsb, cuda, R.SLOT_COUNT)
    for i, batch in enumerate(R.SLOT_STEPS):
        _mark_in_use(cache, i)
        assert _call(cache, batch) == int(d[f"raised{i}"]), i
        active, lens, selected = _state(cache)
        assert active == d[f"active{i}"].tolist(), i
        assert lens == d[f"working_lens{i}"].tolist(), i
        assert selected == np.flatnonzero(d[f"selected{i}"]).tolist(), i
    torch.cuda.synchronize()
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0


@pytest.mark.parametrize("slots,pool,steps", [(64, 120, 300), (7, 12, 200), (1024, 1500, 40)])
def test_slots_match_oracle_random_batches(dsb, cuda, slots, pool, steps):
    rng = random.Random(slots * 1000 + pool)
    ids = [f"req-{k}" for k in range(pool)]
    cache = _cache(dsb, cuda, slots)
    table = O.SlotTable(slots)
    prev: list[str] = []
    for i in range(steps):
        # keep part of the previous batch (shuffled), add new or returning
        # ids, sometimes a duplicate, now and then more than the slots hold
        keep = [r for r in prev if rng.random() < 0.7]
        grow = rng.randint(0, max(1, slots // 3)) if rng.random() < 0.9 else slots + 2
        batch = keep + rng.sample(ids, min(pool, grow))
        if batch and rng.random() < 0.2:
            batch.insert(rng.randrange(len(batch) + 1), rng.choice(batch))
        rng.shuffle(batch)
        _mark_in_use(cache, i)
        for slot in table.slots.values():
            table.working_lens[slot] = 100 + 10 * i + slot
            table.selected.add(slot)
        raised = 0
        try:
            table.set_active_requests(batch)
        except RuntimeError:
            raised = 1
        assert _call(cache, batch) == raised, i
        active, lens, selected = _state(cache)
        assert active == table.active, i
        assert lens == table.working_lens, i
        assert selected == sorted(table.selected), i
        if not raised:
            prev = batch
    torch.cuda.synchronize()
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0


def test_assign_status_and_bad_keys(dsb, cuda):
    """The C entry point alone: status words, a full table, a negative key."""
    lib = dsb._lib.load()
    keys = torch.full((4,), -1, dtype=torch.int64, device=cuda)
    out = torch.empty(6, dtype=torch.int32, device=cuda)
    status = torch.zeros(2, dtype=torch.int32, device=cuda)
    flag = dsb._lib.error_flag(cuda)
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda).cuda_stream)

    def assign(reqs):
        req = torch.tensor(reqs, dtype=torch.int64, device=cuda)
        assert lib.dsb_assign_request_slots(
            ctypes.c_void_p(keys.data_ptr()), 4, ctypes.c_void_p(req.data_ptr()), len(reqs),
            ctypes.c_void_p(out.data_ptr()), None, None, ctypes.c_void_p(status.data_ptr()),
            ctypes.c_void_p(flag.data_ptr()), stream) == 0
        torch.cuda.synchronize()
        return out[: len(reqs)].tolist(), status.tolist(), keys.tolist()

    assert assign([7, 9]) == ([0, 1], [0, 2], [7, 9, -1, -1])
    # 9 kept, 7 released; 5 new keys for 3 free slots: two left without one
    assert assign([11, 9, 12, 13, 14, 15]) == ([0, 1, 2, 3, -1, -1], [2, 0], [11, 9, 12, 13])
    assert dsb._lib.read_and_clear_error_flag(cuda) == 0
    assert assign([9, -5]) == ([1, -1], [0, 3], [-1, 9, -1, -1])
    assert dsb._lib.read_and_clear_error_flag(cuda) == dsb._lib.DSB_FLAG_SLOT


def test_rows_to_slots(dsb, cuda):
    lib = dsb._lib.load()
    active = torch.tensor([5, 2, 7], dtype=torch.int32, device=cuda)
    rows = torch.tensor([0, 0, 2, 1, 3, -1], dtype=torch.int32, device=cuda)
    out = torch.empty(6, dtype=torch.int32, device=cuda)
    flag = dsb._lib.error_flag(cuda)
    assert lib.dsb_rows_to_slots(ctypes.c_void_p(active.data_ptr()), 3,
                                 ctypes.c_void_p(rows.data_ptr()), 6,
                                 ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(flag.data_ptr()),
                                 ctypes.c_void_p(torch.cuda.current_stream(cuda).cuda_stream)) == 0
    assert out.tolist() == [5, 5, 7, 2, -1, -1]
    assert dsb._lib.read_and_clear_error_flag(cuda) == dsb._lib.DSB_FLAG_SLOT
