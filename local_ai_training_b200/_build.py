"""Builds libratchet_b200.so (sm_100a) in-tree with nvcc.

The library has no torch dependency: one compilation unit (csrc/ratchet_b200.cu), static CUDA
runtime, driver entry points fetched at run time (no -lcuda).  The built file lands next to this
module so that it travels with the source tree.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
CSRC = PACKAGE_DIR / "csrc"
LIB_NAME = "libratchet_b200.so"
LIB_PATH = PACKAGE_DIR / LIB_NAME
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    candidate = Path(cuda_home) / "bin" / "nvcc"
    if candidate.exists():
        return str(candidate)
    found = shutil.which("nvcc")
    if found is None:
        raise RuntimeError("nvcc not found; set CUDA_HOME")
    return found


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + [
        PACKAGE_DIR.parent / "include" / "ratchet_b200.h"
    ]


def is_stale() -> bool:
    if not LIB_PATH.exists():
        return True
    built = LIB_PATH.stat().st_mtime
    return any(src.stat().st_mtime > built for src in sources())


def build(*, force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    """Compiles the library if any source is newer than the built file; returns its path."""
    if not force and not is_stale():
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [
        nvcc_path(),
        *ARCH_FLAGS,
        "-lineinfo",
        "-O3",
        "-std=c++17",
        "-DNDEBUG",
        "--expt-relaxed-constexpr",
        "-Xcompiler",
        "-fPIC,-O2",
        "-shared",
        "-cudart",
        "static",
        "-o",
        str(tmp),
        str(CSRC / "ratchet_b200.cu"),
    ]
    if ptxas_info:
        cmd.insert(1, "-Xptxas=-v")
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed ({result.returncode}):\n{result.stderr[-8000:]}")
    if verbose or ptxas_info:
        print(result.stderr, file=sys.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_info="--ptxas-info" in sys.argv)
