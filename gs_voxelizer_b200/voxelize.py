"""Differentiable voxelization of projected Gaussians.

Drop-in for gs_voxelizer/voxelize.py:14-173 of the reference: same function,
arguments, output [Z,Y,X,C], empty-input handling and backward variants
(use_per_gaussian_backward selects the per-Gaussian or the per-voxel CUDA
kernel).
"""
from __future__ import annotations

from typing import Tuple

import torch
from torch import Tensor
from torch.autograd import Function

from . import cuda as _C
from .bin_and_sort_gaussians import bin_and_sort_gaussians


def voxelize_gaussians(
    pos3d_radii: Tensor,
    conics: Tensor,
    intensities: Tensor,
    vol_size_voxel: Tuple[int, int, int],
    tile_min: Tensor,
    tile_max: Tensor,
    num_tiles_hit: Tensor,
    use_per_gaussian_backward: bool = True,
) -> Tensor:
    """Voxelize 3D Gaussians into a [depth, height, width, channels] grid.

    Args:
        pos3d_radii: [N,4] voxel-space positions (xyz) and radii (w).
        conics: [N,6] inverse covariances (a, b, c, d, e, f).
        intensities: [N,C] or [N] intensities, C <= 4.
        vol_size_voxel: (depth, height, width) of the output volume.
        tile_min, tile_max, num_tiles_hit: tile boxes from optim_to_render.
        use_per_gaussian_backward: per-Gaussian backward kernel if True,
            per-voxel kernel otherwise.
    """
    return _VoxelizeGaussians.apply(
        pos3d_radii.contiguous(),
        conics.contiguous(),
        intensities.contiguous(),
        vol_size_voxel,
        tile_min,
        tile_max,
        num_tiles_hit,
        use_per_gaussian_backward,
    )


class _VoxelizeGaussians(Function):
    @staticmethod
    def forward(ctx, pos3d_radii, conics, intensities, vol_size_voxel,
                tile_min, tile_max, num_tiles_hit,
                use_per_gaussian_backward=False):
        ctx.intensity_1d = intensities.dim() == 1
        if ctx.intensity_1d:
            intensities = intensities.unsqueeze(-1)
        num_gaussians = pos3d_radii.size(-2)
        ctx.vol_size_voxel = vol_size_voxel
        ctx.use_per_gaussian_backward = use_per_gaussian_backward
        dev = pos3d_radii.device
        num_intersects = 0
        if num_gaussians > 0:
            cum_tiles_hit = torch.cumsum(num_tiles_hit, dim=0, dtype=torch.int32)
            num_intersects = int(cum_tiles_hit[-1].item())
        ctx.num_intersects = num_intersects
        if num_intersects < 1:
            out = torch.zeros(*vol_size_voxel, intensities.shape[-1],
                              device=dev, dtype=pos3d_radii.dtype)
            ids = torch.zeros(0, 1, device=dev, dtype=torch.int32)
            bins = torch.zeros(0, 3, device=dev, dtype=torch.int32)
        else:
            ids, bins = bin_and_sort_gaussians(
                num_gaussians, num_intersects, tile_min, tile_max,
                cum_tiles_hit, vol_size_voxel)
            out = _C.voxelize_forward(vol_size_voxel, ids, bins, pos3d_radii,
                                      conics, intensities)
        ctx.save_for_backward(pos3d_radii, conics, intensities, ids, bins)
        return out

    @staticmethod
    def backward(ctx, vol_grad):
        pos3d_radii, conics, intensities, ids, bins = ctx.saved_tensors
        if ctx.num_intersects < 1:
            pos_grad = torch.zeros_like(pos3d_radii)
            conics_grad = torch.zeros_like(conics)
            int_grad = torch.zeros_like(intensities)
        else:
            fn = (_C.voxelize_backward_per_gaussian
                  if ctx.use_per_gaussian_backward else _C.voxelize_backward)
            pos_grad, conics_grad, int_grad = fn(
                ctx.vol_size_voxel, ids, bins, pos3d_radii, conics,
                intensities, vol_grad.contiguous())
        if ctx.intensity_1d:
            int_grad = int_grad.reshape(-1)
        return pos_grad, conics_grad, int_grad, None, None, None, None, None
