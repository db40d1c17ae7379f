"""Shared test setup: import paths, the `gpu` marker and fixture loaders."""

from __future__ import annotations

import importlib
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
for p in (str(ROOT), str(GOLDEN)):
    if p not in sys.path:
        sys.path.insert(0, p)

PACKAGE = "vllm-ascend-hust-diffspec_b200"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: runs CUDA kernels; needs an NVIDIA B200 (sm_100a)")


def load_package():
    return importlib.import_module(PACKAGE)


def golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as f:
        return {k: f[k] for k in f.files}


def from_bits(d: dict, key: str) -> np.ndarray:
    """Fixture array as float32 (bf16 keys are stored as uint16 bit patterns)."""
    from oracle.diffspec_oracle import bf16_bits_to_f32

    if key + "_bf16" in d:
        return bf16_bits_to_f32(d[key + "_bf16"])
    if key + "_f16" in d:
        return d[key + "_f16"].astype(np.float32)
    return d[key].astype(np.float32)


def close_bf16(actual: np.ndarray, expected: np.ndarray, max_rel: float = 2e-2,
               mean_rel: float = 2e-3) -> None:
    """The bf16 tolerance of the path: max |a - e| <= 2e-2 * max(1, max|e|)
    and mean |a - e| <= 2e-3 * mean|e| (NaN must match NaN)."""
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    assert a.shape == e.shape, (a.shape, e.shape)
    nan_a, nan_e = np.isnan(a), np.isnan(e)
    assert (nan_a == nan_e).all(), "NaN pattern differs"
    a, e = a[~nan_e], e[~nan_e]
    if e.size == 0:
        return
    err = np.abs(a - e)
    scale = max(1.0, float(np.abs(e).max()))
    assert err.max() <= max_rel * scale, f"max abs err {err.max():.3g} > {max_rel * scale:.3g}"
    denom = max(float(np.abs(e).mean()), 1e-12)
    assert err.mean() <= mean_rel * denom, f"mean err {err.mean():.3g} > {mean_rel * denom:.3g}"


@pytest.fixture(scope="session")
def dsb():
    return load_package()


@pytest.fixture(scope="session")
def cuda():
    """The CUDA device for `gpu` tests; fails (never skips) without one."""
    import torch

    assert torch.cuda.is_available(), "gpu tests need a CUDA device (there is no CPU path)"
    return torch.device("cuda", 0)
