"""ctypes binding of libgsvox.so, the C ABI declared in include/gsvox.h.

The library is built in-tree by ``gs_voxelizer_b200/build.py`` (or
``__graft_entry__.build()``). There is no fallback: if the shared library is
missing or fails to load, importing this module raises ImportError.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

_PATH = Path(os.environ.get("GSVOX_LIB", Path(__file__).resolve().parent / "libgsvox.so"))

if not _PATH.exists():
    raise ImportError(
        f"libgsvox.so not found at {_PATH}; build it with "
        "`python gs_voxelizer_b200/build.py` (nvcc, sm_100a)")

lib = ctypes.CDLL(str(_PATH))

_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64
_SZ = ctypes.c_size_t
_I3 = ctypes.c_int32 * 3
_F3 = ctypes.c_float * 3

# name -> (restype, argtypes); kept in declaration order of include/gsvox.h
SIGNATURES = {
    "gsv_last_error": (ctypes.c_char_p, []),
    "gsv_version": (ctypes.c_char_p, []),
    "gsv_launch_count": (ctypes.c_uint64, []),
    "gsv_profile_kernel": (ctypes.c_int, [_I32, _P, _P]),
    "gsv_set_tensor_core_backward": (ctypes.c_int, [_I32]),
    "gsv_device_error": (ctypes.c_int, [_P, _I32]),
    "gsv_ssim3d_workspace_bytes": (ctypes.c_size_t, [_I32, _P]),
    "gsv_ssim3d_forward": (ctypes.c_int, [_I32, _P, _P, _P, ctypes.c_float,
                                          ctypes.c_float, _P, _P, ctypes.c_size_t, _P]),
    "gsv_ssim3d_backward": (ctypes.c_int, [_I32, _P, _P, _P, _P, _P,
                                           ctypes.c_size_t, _P, _P]),
    "gsv_tv3d_workspace_bytes": (ctypes.c_size_t, [_I32, _P]),
    "gsv_tv3d": (ctypes.c_int, [_I32, _P, _P, _I32, ctypes.c_float, _P, _P, _P,
                                _P, ctypes.c_size_t, _P]),
    "gsv_optim_to_render_forward": (
        ctypes.c_int, [_I32, _I32, _P, _P, _P, _P, _I3, _F3, _F3,
                       _P, _P, _P, _P, _P, _P]),
    "gsv_optim_to_render_backward": (
        ctypes.c_int, [_I32, _P, _P, _P, _I3, _F3, _F3, _P, _P, _P,
                       _P, _P, _P, _P]),
    "gsv_bin_and_sort_workspace_bytes": (_SZ, [_I32, _I64, _I3]),
    "gsv_bin_and_sort_gaussians": (
        ctypes.c_int, [_I32, _I64, _P, _P, _P, _I3, _P, _P, _P, _SZ, _P]),
    "gsv_bin_and_sort_slab_workspace_bytes": (_SZ, [_I32, _I64, _I3, _I32, _I32]),
    "gsv_bin_and_sort_gaussians_slab": (
        ctypes.c_int, [_I32, _I64, _P, _P, _I3, _I32, _I32, _P, _P, _P, _SZ, _P]),
    "gsv_count_slab_intersects": (
        ctypes.c_int, [_I32, _P, _P, _I32, _I32, _P, _P]),
    "gsv_voxelize_workspace_bytes": (_SZ, [_I32, _I32, _I64, _I3]),
    "gsv_voxelize_forward": (
        ctypes.c_int, [_I3, _I32, _I32, _I64, _P, _P, _P, _P, _P, _P,
                       _P, _SZ, _P]),
    "gsv_voxelize_backward_per_gaussian": (
        ctypes.c_int, [_I3, _I32, _I32, _I64, _P, _P, _P, _P, _P, _P,
                       _P, _P, _P, _P, _SZ, _P]),
    "gsv_voxelize_backward": (
        ctypes.c_int, [_I3, _I32, _I32, _I64, _P, _P, _P, _P, _P, _P,
                       _P, _P, _P, _P, _SZ, _P]),
    "gsv_voxelize_slab_workspace_bytes": (_SZ, [_I32, _I32, _I64, _I3, _I32, _I32]),
    "gsv_voxelize_forward_slab": (
        ctypes.c_int, [_I3, _I32, _I32, _I32, _I32, _I64, _P, _P, _P, _P, _P,
                       _P, _P, _SZ, _P]),
    "gsv_voxelize_backward_per_gaussian_slab": (
        ctypes.c_int, [_I3, _I32, _I32, _I32, _I32, _I64, _P, _P, _P, _P, _P,
                       _P, _P, _P, _P, _P, _SZ, _P]),
    "gsv_l1_loss_workspace_bytes": (_SZ, [_I64]),
    "gsv_l1_loss_forward": (
        ctypes.c_int, [_I64, _P, _P, ctypes.c_float, _P, _P, _SZ, _P]),
    "gsv_l1_loss_backward": (
        ctypes.c_int, [_I64, _P, _P, _P, ctypes.c_float, _P, _P]),
    "gsv_voxelize_l1_workspace_bytes": (_SZ, [_I32, _I32, _I64, _I3, _I32, _I32]),
    "gsv_voxelize_forward_l1": (
        ctypes.c_int, [_I3, _I32, _I32, _I32, _I32, _I64, _P, _P, _P, _P, _P,
                       _P, ctypes.c_float, _P, _P, _P, _P, _P, _P, _P, _SZ,
                       _P]),
    "gsv_voxelize_backward_per_gaussian_l1": (
        ctypes.c_int, [_I3, _I32, _I32, _I32, _I32, _I64, _P, _P, _P, _P, _P,
                       _P, _P, _P, ctypes.c_float, _P, _P, _P, _P, _SZ, _P]),
    "gsv_voxelize_forward_noalloc": (
        ctypes.c_int, [_I3, _I32, _I32, _I64, _P, _P, _P, _P, _P, _P, _P]),
    "gsv_halo_workspace_bytes": (_SZ, [_I32, _I32]),
    "gsv_halo_pack": (
        ctypes.c_int, [_I32, _I32, _P, _P, _P, _P, _P, _I32, _I32, _P, _P, _P,
                       _P, _P, _P, _P, _SZ, _P]),
    "gsv_halo_unpack": (
        ctypes.c_int, [_I32, _I32, _I32, _I32, _P, _P, _P, _P, _P, _P, _P, _P,
                       _P, _P]),
    "gsv_peer_barrier": (ctypes.c_int, [_I32, _I32, _P, _P, _P]),
    "gsv_halo_pack_peers": (
        ctypes.c_int, [_I32, _I32, _P, _P, _P, _P, _P, _I32, _I32, _P, _P, _P,
                       _P, _P, _P, _P, _SZ, _P]),
    "gsv_halo_pack_grads_peers": (
        ctypes.c_int, [_I32, _I32, _I32, _I32, _P, _P, _P, _P, _P, _P, _P, _P,
                       _P]),
    "gsv_halo_pack_grads": (
        ctypes.c_int, [_I32, _I32, _I32, _I32, _P, _P, _P, _P, _P, _P, _P, _P,
                       _P]),
    "gsv_halo_accumulate": (
        ctypes.c_int, [_I32, _I32, _I32, _I32, _P, _P, _P, _P, _P, _P, _P, _P,
                       _P, _P]),
}

HALO_RECORD_FLOATS = 20
HALO_GRAD_FLOATS = 16

for _name, (_res, _args) in SIGNATURES.items():
    _fn = getattr(lib, _name)
    _fn.restype = _res
    _fn.argtypes = _args

STATUS = {
    0: "GSV_OK",
    1: "GSV_ERR_INVALID_ARGUMENT",
    2: "GSV_ERR_UNSUPPORTED_CHANNELS",
    3: "GSV_ERR_WORKSPACE_TOO_SMALL",
    4: "GSV_ERR_SIZE_OVERFLOW",
    5: "GSV_ERR_CUDA",
}


class GsvError(RuntimeError):
    """A libgsvox call returned a non-zero status."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS.get(status, status)}: {message}")
        self.status = status


def check(status: int) -> None:
    if status != 0:
        msg = lib.gsv_last_error().decode(errors="replace")
        raise GsvError(status, msg)


def i3(t) -> ctypes.Array:
    return _I3(*(int(v) for v in t))


def f3(t) -> ctypes.Array:
    return _F3(*(float(v) for v in t))


def version() -> str:
    return lib.gsv_version().decode()
