"""Build libgsvox.so (the C-ABI library of include/gsvox.h) in-tree with nvcc.

sm_100a only: every translation unit is compiled with
``-gencode arch=compute_100a,code=sm_100a``. Object files go to ``_build/``
beside this file; the shared library lands next to the package sources so
that it travels with the repository snapshot.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "csrc"
BUILD = HERE / "_build"
LIB = HERE / "libgsvox.so"
SOURCES = ["projection.cu", "binning.cu", "voxelize.cu", "bwd_tc.cu", "loss.cu",
           "ssim.cu", "noalloc.cu", "halo.cu", "capi.cu"]

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# -use_fast_math matches the reference's build (setup.py:139), which the
# projection's bit-exact tile bounds depend on.
FLAGS = ["-O3", "-lineinfo", "-use_fast_math", "-std=c++17",
         "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
         "-Xcompiler", "-fvisibility=hidden"]


def _run(cmd: list[str]) -> None:
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"command failed: {' '.join(cmd)}")


def build(verbose: bool = False, ptxas_info: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    deps = [SRC / "common.cuh", HERE.parent / "include" / "gsvox.h"]
    dep_mtime = max(p.stat().st_mtime for p in deps)
    objs = []
    for name in SOURCES:
        src = SRC / name
        obj = BUILD / (name + ".o")
        objs.append(obj)
        if obj.exists() and obj.stat().st_mtime > max(src.stat().st_mtime, dep_mtime) \
                and not ptxas_info:
            continue
        cmd = [NVCC, *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
        if ptxas_info:
            cmd.insert(1, "-Xptxas=-v")
        if verbose:
            print(" ".join(cmd))
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            sys.stderr.write(res.stdout + res.stderr)
            raise RuntimeError(f"nvcc failed on {name}")
        if ptxas_info:
            sys.stdout.write(res.stderr)
    if not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        _run([NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs),
              "-Xcompiler", "-fPIC", "-cudart", "static"])
    return LIB


if __name__ == "__main__":
    build(verbose=True, ptxas_info="-v" in sys.argv)
    print(LIB)
