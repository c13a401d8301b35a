"""Build the C oracle (test infrastructure): oracle/_ref/libhvoracle.so.

    python oracle/build_oracle.py

gcc -O3 -fopenmp -ffp-contract=off: no fused multiply-adds, so every float operation
rounds the way numpy's does. The output directory is git-ignored; the library is
rebuilt from source wherever the tests run.
"""
from __future__ import annotations

import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
LIB = OUT / "libhvoracle.so"
SRC = HERE / "hv_oracle_c.c"


def build(force: bool = False) -> Path:
    if not force and LIB.exists() and LIB.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB
    OUT.mkdir(exist_ok=True)
    cmd = ["gcc", "-O3", "-fopenmp", "-ffp-contract=off", "-fno-fast-math", "-fPIC",
           "-shared", "-o", str(LIB), str(SRC), "-lm"]
    subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
