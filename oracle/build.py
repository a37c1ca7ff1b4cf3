"""Build the CPU oracle (TEST INFRASTRUCTURE: the checker and CPU baseline only).

    python -m oracle.build

Compiles oracle/ksd8_oracle.c with gcc into oracle/_ref/libksd8_oracle.so
(FMA contraction off so fp32 expressions round as written; OpenMP for the
multi-core CPU baseline).  Nothing in the ksdraft_b200 product imports this.
"""

from __future__ import annotations

import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "ksd8_oracle.c"
OUT_DIR = HERE / "_ref"
LIB = OUT_DIR / "libksd8_oracle.so"


def build(force: bool = False) -> Path:
    OUT_DIR.mkdir(exist_ok=True)
    if force or not LIB.exists() or LIB.stat().st_mtime < SRC.stat().st_mtime:
        cmd = ["gcc", "-O2", "-std=c11", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off",
               "-fno-fast-math", "-Wall", "-o", str(LIB), str(SRC), "-lm"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"oracle build failed:\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(force=True))
