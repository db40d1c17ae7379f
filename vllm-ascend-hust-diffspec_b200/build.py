"""Build libdiffspec_b200.so (sm_100a) in-tree with nvcc.

The library is plain CUDA C++ behind the C ABI declared in
include/diffspec_b200.h; it links the CUDA runtime statically and has no
PyTorch dependency.  Objects go to _build/ under the repository root; the
shared object is written next to this file so it travels with the package.

Usage: python vllm-ascend-hust-diffspec_b200/build.py [--force] [--verbose-ptxas]
"""

from __future__ import annotations

import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_ROOT = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
INCLUDE = REPO_ROOT / "include"
BUILD_DIR = REPO_ROOT / "_build" / "diffspec_b200"
LIB_NAME = "libdiffspec_b200.so"
LIB_PATH = PKG_DIR / LIB_NAME

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "--expt-relaxed-constexpr",
    "-I",
    str(INCLUDE),
    "-I",
    str(CSRC),
]


def _nvcc() -> str:
    candidates = [
        os.environ.get("NVCC"),
        shutil.which("nvcc"),
        "/usr/local/cuda/bin/nvcc",
    ]
    for cand in candidates:
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the DiffSpec B200 library needs the CUDA toolkit")


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    mtime = target.stat().st_mtime
    return any(dep.stat().st_mtime > mtime for dep in deps)


def _compile(nvcc: str, src: Path, verbose_ptxas: bool) -> Path:
    obj = BUILD_DIR / (src.stem + ".o")
    cmd = [nvcc, *ARCH_FLAGS, *COMMON_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{proc.stdout}\n{proc.stderr}")
    if verbose_ptxas:
        sys.stderr.write(proc.stderr)
    return obj


def build(force: bool = False, verbose_ptxas: bool = False) -> Path:
    """Compile every kernel source for sm_100a and link the shared library."""
    nvcc = _nvcc()
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    sources = _sources()
    headers = _headers()
    todo = [
        src
        for src in sources
        if force or verbose_ptxas or _stale(BUILD_DIR / (src.stem + ".o"), [src, *headers])
    ]
    if todo:
        workers = min(len(todo), os.cpu_count() or 4)
        with concurrent.futures.ThreadPoolExecutor(workers) as pool:
            list(pool.map(lambda s: _compile(nvcc, s, verbose_ptxas), todo))
    objects = [BUILD_DIR / (src.stem + ".o") for src in sources]
    if force or todo or _stale(LIB_PATH, objects):
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objects)]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link failed:\n{proc.stdout}\n{proc.stderr}")
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose-ptxas", action="store_true")
    args = parser.parse_args()
    print(build(force=args.force, verbose_ptxas=args.verbose_ptxas))


if __name__ == "__main__":
    main()
