"""Compiles the CPU oracle (ratchet_oracle.c) with gcc into oracle/libratchet_oracle.so.

Strict IEEE fp32 semantics: no fast-math, no FMA contraction, SSE arithmetic.
"""

from __future__ import annotations

import os
import subprocess
from pathlib import Path

ORACLE_DIR = Path(__file__).resolve().parent
SOURCE = ORACLE_DIR / "ratchet_oracle.c"
LIB_PATH = ORACLE_DIR / "libratchet_oracle.so"


def build(force: bool = False) -> Path:
    if not force and LIB_PATH.exists() and LIB_PATH.stat().st_mtime >= SOURCE.stat().st_mtime:
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = ["gcc", "-O2", "-std=c11", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared",
           "-o", str(tmp), str(SOURCE), "-lm"]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{result.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force=True))
