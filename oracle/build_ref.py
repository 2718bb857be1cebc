"""Compile the reference's own CUDA extension (PaPieta/gs-voxelizer,
gs_voxelizer/cuda/*.cu + ext.cpp) for sm_100a into oracle/_ref/.

Parity oracle only: tests and the bench's reference arm load the result;
the product never does. The sources are compiled where they lie (read-only,
never copied); GLM, which the reference downloads at build time
(setup.py:43-66) and which is absent here, is replaced by the header shim in
oracle/glm_shim. Flags follow the reference's setup.py:137-149 (-O3
--use_fast_math --expt-relaxed-constexpr) plus the sm_100a target.

Usage: python oracle/build_ref.py [REFERENCE_ROOT]
REFERENCE_ROOT defaults to $GSV_REFERENCE_ROOT, else a directory named
`reference` beside the repository's own directory.
Output: oracle/_ref/gs_voxelizer_ref_cuda*.so (git-ignored; it travels to the
GPU box with the repository snapshot).
"""
from __future__ import annotations

import glob
import os
import shutil
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
NAME = "gs_voxelizer_ref_cuda"


def built_library() -> Path | None:
    hits = sorted(OUT.glob(f"{NAME}*.so"))
    return hits[0] if hits else None


def default_root() -> str:
    """$GSV_REFERENCE_ROOT, else `reference` beside the repository."""
    return os.environ.get("GSV_REFERENCE_ROOT",
                          str(HERE.parent.parent / "reference"))


def build(reference_root: str | None = None) -> Path | None:
    reference_root = reference_root or default_root()
    src_dir = Path(reference_root) / "gs_voxelizer" / "cuda"
    if not src_dir.is_dir():
        return built_library()
    sources = sorted(glob.glob(str(src_dir / "*.cu"))) + sorted(glob.glob(str(src_dir / "*.cpp")))
    newest = max(os.path.getmtime(s) for s in sources)
    lib = built_library()
    if lib is not None and lib.stat().st_mtime > newest:
        return lib
    from torch.utils.cpp_extension import load

    build_dir = OUT / "build"
    build_dir.mkdir(parents=True, exist_ok=True)
    os.environ.setdefault("MAX_JOBS", str(min(8, os.cpu_count() or 1)))
    load(
        name=NAME,
        sources=sources,
        extra_include_paths=[str(HERE / "glm_shim")],
        extra_cflags=["-O3", "-Wno-sign-compare"],
        extra_cuda_cflags=["-O3", "--use_fast_math", "--expt-relaxed-constexpr",
                           "-gencode=arch=compute_100a,code=sm_100a"],
        build_directory=str(build_dir),
        verbose=False,
        is_python_module=True,
    )
    so = sorted(build_dir.glob(f"{NAME}*.so"))
    if not so:
        raise RuntimeError("reference extension build produced no .so")
    dst = OUT / so[0].name
    shutil.copy2(so[0], dst)
    return dst


def load_reference():
    """Import the built reference extension module (torch must be importable)."""
    import importlib.util

    import torch  # noqa: F401  (the extension links against libtorch)

    lib = built_library()
    if lib is None:
        return None
    spec = importlib.util.spec_from_file_location(NAME, str(lib))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else default_root()
    print(build(root))
