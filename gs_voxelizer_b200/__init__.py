"""B200-native (sm_100a) differentiable Gaussian voxelization.

Drop-in for the Python API of PaPieta/gs-voxelizer: the submodules
``optim_to_render``, ``voxelize`` and ``bin_and_sort_gaussians`` carry the
same functions, and ``cuda`` the six extension entry points. The kernels live
in libgsvox.so (C ABI: include/gsvox.h), built by ``build.py``.
"""
__version__ = "0.1.0"
