"""Build the CPU oracle (gsv_oracle.c) into oracle/_build/liboracle.so.

Test infrastructure only: the library is the checker of the parity tests,
smoke() and bench.py's cpu_baseline leg; the product never links it.
-ffp-contract=off keeps the float arithmetic in source order (no fused
multiply-add), the IEEE reading of the reference's expressions.
"""
from __future__ import annotations

import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "gsv_oracle.c"
OUT = HERE / "_build" / "liboracle.so"


def build() -> Path:
    OUT.parent.mkdir(exist_ok=True)
    if OUT.exists() and OUT.stat().st_mtime > SRC.stat().st_mtime:
        return OUT
    cmd = ["gcc", "-O3", "-march=x86-64-v2", "-ffp-contract=off", "-fopenmp",
           "-fPIC", "-shared", "-std=c11", str(SRC), "-o", str(OUT), "-lm"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("building the CPU oracle failed")
    return OUT


if __name__ == "__main__":
    print(build())
