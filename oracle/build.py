"""Build oracle/liboracle.so from kb_oracle.c (test infrastructure only).

Compiled without FMA contraction or fast-math so every float operation is a
single IEEE rounding, as in the kernels it checks.
"""
from __future__ import annotations

import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "kb_oracle.c"
LIB = HERE / "liboracle.so"


def build(force: bool = False) -> Path:
    if not force and LIB.exists() and LIB.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = ["gcc", "-O2", "-fPIC", "-shared", "-ffp-contract=off", "-fno-fast-math",
           "-std=c11", "-Wall", "-o", str(tmp), str(SRC), "-lm"]
    subprocess.run(cmd, check=True)
    tmp.replace(LIB)
    return LIB


if __name__ == "__main__":
    print(build(force=True))
