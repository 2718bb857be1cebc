"""B200-native (sm_100a) differentiable Gaussian voxelization.

Drop-in for the Python API of PaPieta/gs-voxelizer: the submodules
``optim_to_render``, ``voxelize`` and ``bin_and_sort_gaussians`` carry the
same functions, and ``cuda`` the six extension entry points. The kernels live
in libgsvox.so (C ABI: include/gsvox.h), built by ``build.py``.
"""
__version__ = "0.1.0"

_ALIASED = ("optim_to_render", "voxelize", "bin_and_sort_gaussians", "cuda")


def install_alias(name: str = "gs_voxelizer") -> None:
    """Make ``import gs_voxelizer`` (and its submodules ``optim_to_render``,
    ``voxelize``, ``bin_and_sort_gaussians`` and ``cuda``) resolve to this
    package, so that code written against the reference
    (``from gs_voxelizer.voxelize import voxelize_gaussians``, the module
    layout of the reference's setup.py:153-155) runs unchanged. Opt-in: call
    it once before those imports. Raises ImportError if another module of
    that name is already imported."""
    import importlib
    import sys
    existing = sys.modules.get(name)
    if existing is not None and existing is not sys.modules[__name__]:
        raise ImportError(f"a module named {name!r} is already imported")
    sys.modules[name] = sys.modules[__name__]
    for sub in _ALIASED:
        sys.modules[f"{name}.{sub}"] = importlib.import_module(f"{__name__}.{sub}")
