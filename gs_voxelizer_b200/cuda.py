"""Tensor-level entry points with the names and signatures of the reference's
extension module ``gs_voxelizer.cuda`` (gs_voxelizer/cuda/ext.cpp:4-11,
bindings.h:40-194).

Each function checks its tensors the way the reference's CHECK_INPUT does
(bindings.h:7-12: CUDA and contiguous, else RuntimeError), allocates its
outputs and workspace with torch on the input's device, and calls the
matching ``gsv_*`` C-ABI function on torch's current CUDA stream. Outputs are
fully written by the kernels (no separate zeroing pass).
"""
from __future__ import annotations

from typing import Sequence, Tuple

import torch

from . import _lib
from ._lib import check, f3, i3, lib

MAX_CHANNELS = 4
TILE = 8


def _check_input(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


def _check_f32(t: torch.Tensor, name: str) -> None:
    if t.dtype != torch.float32:
        raise RuntimeError(f"{name} must be float32, got {t.dtype}")


def _check_i32(t: torch.Tensor, name: str) -> None:
    if t.dtype != torch.int32:
        raise RuntimeError(f"{name} must be int32, got {t.dtype}")


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None or t.numel() == 0 else t.data_ptr()


def _channels(intensities: torch.Tensor) -> int:
    c = 1 if intensities.dim() == 1 else int(intensities.size(1))
    if c > MAX_CHANNELS:
        raise RuntimeError("Number of channels exceeds MAX_CHANNELS")
    if c < 1:
        raise RuntimeError("Unsupported number of channels")
    return c


def num_tiles(vol_size: Sequence[int]) -> int:
    z, y, x = (int(v) for v in vol_size)
    return ((z + TILE - 1) // TILE) * ((y + TILE - 1) // TILE) * ((x + TILE - 1) // TILE)


def _workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


def optim_to_render_forward(
    num_gaussians: int,
    pos3d: torch.Tensor,
    scale3d: torch.Tensor,
    quat: torch.Tensor,
    intensities: torch.Tensor,
    vol_size_voxel: Tuple[int, int, int],
    vol_size_world: Tuple[float, float, float],
    vol_center_pos: Tuple[float, float, float],
):
    """bindings.cu:44. Returns (pos3d_radii [N,4], conics [N,6],
    tile_min [N,3] int32, tile_max [N,3] int32, num_tiles_hit [N] int32)."""
    for t, n in ((pos3d, "pos3d"), (scale3d, "scale3d"), (quat, "quat"),
                 (intensities, "intensities")):
        _check_input(t, n)
        _check_f32(t, n)
    C = _channels(intensities)
    n = int(num_gaussians)
    dev = pos3d.device
    f = dict(device=dev, dtype=torch.float32)
    i = dict(device=dev, dtype=torch.int32)
    pos3d_radii = torch.empty((n, 4), **f)
    conics = torch.empty((n, 6), **f)
    tile_min = torch.empty((n, 3), **i)
    tile_max = torch.empty((n, 3), **i)
    num_tiles_hit = torch.empty((n,), **i)
    check(lib.gsv_optim_to_render_forward(
        n, C, _ptr(pos3d), _ptr(scale3d), _ptr(quat), _ptr(intensities),
        i3(vol_size_voxel), f3(vol_size_world), f3(vol_center_pos),
        _ptr(pos3d_radii), _ptr(conics), _ptr(tile_min), _ptr(tile_max),
        _ptr(num_tiles_hit), _stream(dev)))
    return pos3d_radii, conics, tile_min, tile_max, num_tiles_hit


def optim_to_render_backward(
    num_gaussians: int,
    pos3d: torch.Tensor,
    scale3d: torch.Tensor,
    quat: torch.Tensor,
    vol_size_voxel: Tuple[int, int, int],
    vol_size_world: Tuple[float, float, float],
    vol_center_pos: Tuple[float, float, float],
    pos3d_radii_grad_in: torch.Tensor,
    conics_grad_in: torch.Tensor,
    pos3d_radii_out: torch.Tensor,
):
    """bindings.cu:201. Returns (pos3d_grad [N,3], scale3d_grad [N,3],
    quat_grad [N,4])."""
    pos3d_radii_grad_in = pos3d_radii_grad_in.contiguous()
    conics_grad_in = conics_grad_in.contiguous()
    for t, name in ((pos3d, "pos3d"), (scale3d, "scale3d"), (quat, "quat"),
                    (pos3d_radii_grad_in, "pos3d_radii_grad_in"),
                    (conics_grad_in, "conics_grad_in"),
                    (pos3d_radii_out, "pos3d_radii_out")):
        _check_input(t, name)
        _check_f32(t, name)
    n = int(num_gaussians)
    dev = pos3d.device
    f = dict(device=dev, dtype=torch.float32)
    pos_grad = torch.empty((n, 3), **f)
    scale_grad = torch.empty((n, 3), **f)
    quat_grad = torch.empty((n, 4), **f)
    check(lib.gsv_optim_to_render_backward(
        n, _ptr(pos3d), _ptr(scale3d), _ptr(quat), i3(vol_size_voxel),
        f3(vol_size_world), f3(vol_center_pos), _ptr(pos3d_radii_grad_in),
        _ptr(conics_grad_in), _ptr(pos3d_radii_out), _ptr(pos_grad),
        _ptr(scale_grad), _ptr(quat_grad), _stream(dev)))
    return pos_grad, scale_grad, quat_grad


def bin_and_sort_gaussians(
    num_gaussians: int,
    num_intersects: int,
    tile_min: torch.Tensor,
    tile_max: torch.Tensor,
    cum_tiles_hit: torch.Tensor,
    vol_size: Tuple[int, int, int],
):
    """bindings.cu:261. Returns (gaussian_ids_sorted [I] int32,
    tile_bins [T,2] int32)."""
    for t, name in ((tile_min, "tile_min"), (tile_max, "tile_max"),
                    (cum_tiles_hit, "cum_tiles_hit")):
        _check_input(t, name)
    _check_i32(tile_min, "tile_min")
    _check_i32(tile_max, "tile_max")
    dev = tile_min.device
    T = num_tiles(vol_size)
    n_isect = max(0, int(num_intersects))
    ids = torch.empty((n_isect,), dtype=torch.int32, device=dev)
    bins = torch.empty((T, 2), dtype=torch.int32, device=dev)
    vol = i3(vol_size)
    ws_bytes = lib.gsv_bin_and_sort_workspace_bytes(int(num_gaussians), n_isect, vol)
    ws = _workspace(ws_bytes, dev)
    check(lib.gsv_bin_and_sort_gaussians(
        int(num_gaussians), n_isect, _ptr(tile_min), _ptr(tile_max),
        _ptr(cum_tiles_hit), vol, _ptr(ids), _ptr(bins), _ptr(ws), ws.numel(),
        _stream(dev)))
    return ids, bins


def _vox_inputs(gaussian_ids_sorted, tile_bins, pos3d, conics, intensities):
    for t, name in ((gaussian_ids_sorted, "gaussian_ids_sorted"),
                    (tile_bins, "tile_bins"), (pos3d, "pos3d"),
                    (conics, "conics"), (intensities, "intensities")):
        _check_input(t, name)
    _check_i32(gaussian_ids_sorted, "gaussian_ids_sorted")
    _check_i32(tile_bins, "tile_bins")
    for t, name in ((pos3d, "pos3d"), (conics, "conics"),
                    (intensities, "intensities")):
        _check_f32(t, name)
    return _channels(intensities)


def voxelize_forward(
    vol_size: Tuple[int, int, int],
    gaussian_ids_sorted: torch.Tensor,
    tile_bins: torch.Tensor,
    pos3d: torch.Tensor,
    conics: torch.Tensor,
    intensities: torch.Tensor,
):
    """bindings.cu:362. Returns the volume [Z,Y,X,C] float32."""
    C = _vox_inputs(gaussian_ids_sorted, tile_bins, pos3d, conics, intensities)
    n = int(pos3d.size(0))
    n_isect = int(gaussian_ids_sorted.numel())
    dev = pos3d.device
    z, y, x = (int(v) for v in vol_size)
    out = torch.empty((z, y, x, C), dtype=torch.float32, device=dev)
    vol = i3(vol_size)
    ws = _workspace(lib.gsv_voxelize_workspace_bytes(n, C, n_isect, vol), dev)
    check(lib.gsv_voxelize_forward(
        vol, C, n, n_isect, _ptr(gaussian_ids_sorted), _ptr(tile_bins),
        _ptr(pos3d), _ptr(conics), _ptr(intensities), _ptr(out), _ptr(ws),
        ws.numel(), _stream(dev)))
    return out


def _backward(fn, vol_size, gaussian_ids_sorted, tile_bins, pos3d, conics,
              intensities, vol_grad_in):
    C = _vox_inputs(gaussian_ids_sorted, tile_bins, pos3d, conics, intensities)
    vol_grad_in = vol_grad_in.contiguous()
    _check_input(vol_grad_in, "vol_grad_in")
    _check_f32(vol_grad_in, "vol_grad_in")
    n = int(pos3d.size(0))
    n_isect = int(gaussian_ids_sorted.numel())
    dev = pos3d.device
    f = dict(device=dev, dtype=torch.float32)
    pos_grad = torch.empty((n, 4), **f)
    conics_grad = torch.empty((n, 6), **f)
    int_grad = torch.empty((n, C), **f)
    vol = i3(vol_size)
    ws = _workspace(lib.gsv_voxelize_workspace_bytes(n, C, n_isect, vol), dev)
    check(fn(vol, C, n, n_isect, _ptr(gaussian_ids_sorted), _ptr(tile_bins),
             _ptr(pos3d), _ptr(conics), _ptr(intensities), _ptr(vol_grad_in),
             _ptr(pos_grad), _ptr(conics_grad), _ptr(int_grad), _ptr(ws),
             ws.numel(), _stream(dev)))
    return pos_grad, conics_grad, int_grad


def voxelize_backward(vol_size, gaussian_ids_sorted, tile_bins, pos3d, conics,
                      intensities, vol_grad_in):
    """bindings.cu:462 (per-voxel work distribution). Returns
    (pos3d_grad [N,4], conics_grad [N,6], intensities_grad [N,C])."""
    return _backward(lib.gsv_voxelize_backward, vol_size, gaussian_ids_sorted,
                     tile_bins, pos3d, conics, intensities, vol_grad_in)


def voxelize_backward_per_gaussian(vol_size, gaussian_ids_sorted, tile_bins,
                                   pos3d, conics, intensities, vol_grad_in):
    """bindings.cu:589 (per-Gaussian work distribution). Returns
    (pos3d_grad [N,4], conics_grad [N,6], intensities_grad [N,C])."""
    return _backward(lib.gsv_voxelize_backward_per_gaussian, vol_size,
                     gaussian_ids_sorted, tile_bins, pos3d, conics,
                     intensities, vol_grad_in)


__all__ = [
    "optim_to_render_forward",
    "optim_to_render_backward",
    "bin_and_sort_gaussians",
    "voxelize_forward",
    "voxelize_backward",
    "voxelize_backward_per_gaussian",
]
_ = _lib
