"""Projection of optimisation parameters to render parameters.

Drop-in for gs_voxelizer/optim_to_render.py:12-149 of the reference: same
function, arguments, outputs, autograd behaviour (no gradient to intensities
through this step) and ValueError checks.
"""
from __future__ import annotations

from typing import Optional, Tuple

from torch import Tensor
from torch.autograd import Function

from . import cuda as _C


def optim_to_render(
    pos3d: Tensor,
    scale3d: Tensor,
    quat: Tensor,
    intensities: Tensor,
    vol_size_voxel: Tuple[int, int, int],
    vol_size_world: Tuple[float, float, float],
    vol_center_pos: Tuple[float, float, float],
    pos3d_radii_buffer: Optional[Tensor] = None,
) -> Tuple[Tensor, Tensor, Tensor, Tensor, Tensor]:
    """Convert Gaussians from optimisation parameters to render parameters.

    Args:
        pos3d: [N,3] positions in world units (x, y, z).
        scale3d: [N,3] per-axis scales in world units.
        quat: [N,4] quaternions (w, x, y, z).
        intensities: [N,C] (or [N]) intensities, C <= 4.
        vol_size_voxel: (depth, height, width) in voxels.
        vol_size_world: (depth, height, width) in world units.
        vol_center_pos: (z, y, x) volume centre in world units.
        pos3d_radii_buffer: optional preallocated contiguous [N,4] tensor
            that receives the returned positions/radii.

    Returns:
        pos3d_radii [N,4] (voxel-space x, y, z and cull radius in w),
        conics [N,6], tile_min [N,3], tile_max [N,3], num_tiles_hit [N].
    """
    return _OptimToRender.apply(
        pos3d.contiguous(),
        scale3d.contiguous(),
        quat.contiguous(),
        intensities.contiguous(),
        vol_size_voxel,
        vol_size_world,
        vol_center_pos,
        pos3d_radii_buffer,
    )


class _OptimToRender(Function):
    @staticmethod
    def forward(ctx, pos3d, scale3d, quat, intensities, vol_size_voxel,
                vol_size_world, vol_center_pos, pos3d_radii_buffer):
        num_gaussians = pos3d.size(-2)
        if num_gaussians < 1 or pos3d.shape[-1] != 3:
            raise ValueError(f"Invalid shape for pos3d: {pos3d.shape}")
        pos3d_radii, conics, tile_min, tile_max, num_tiles_hit = \
            _C.optim_to_render_forward(num_gaussians, pos3d, scale3d, quat,
                                       intensities, vol_size_voxel,
                                       vol_size_world, vol_center_pos)
        ctx.num_gaussians = num_gaussians
        ctx.vol_size_voxel = vol_size_voxel
        ctx.vol_size_world = vol_size_world
        ctx.vol_center_pos = vol_center_pos
        ctx.save_for_backward(pos3d, scale3d, quat, pos3d_radii)
        ctx.mark_non_differentiable(tile_min, tile_max, num_tiles_hit)

        if pos3d_radii_buffer is not None:
            if not pos3d_radii_buffer.is_contiguous():
                raise ValueError("pos3d_radii_buffer must be contiguous")
            if pos3d_radii_buffer.shape != pos3d_radii.shape:
                raise ValueError(
                    "pos3d_radii_buffer shape mismatch: expected "
                    f"{pos3d_radii.shape}, got {pos3d_radii_buffer.shape}")
            if pos3d_radii_buffer.device != pos3d_radii.device:
                raise ValueError("pos3d_radii_buffer must be on the same device as inputs")
            if pos3d_radii_buffer.dtype != pos3d_radii.dtype:
                raise ValueError("pos3d_radii_buffer must share dtype with inputs")
            pos3d_radii_buffer.copy_(pos3d_radii)
            pos3d_radii = pos3d_radii_buffer
        return pos3d_radii, conics, tile_min, tile_max, num_tiles_hit

    @staticmethod
    def backward(ctx, pos3d_radii_grad, conics_grad, _tmin_g, _tmax_g, _nt_g):
        pos3d, scale3d, quat, pos3d_radii = ctx.saved_tensors
        if pos3d_radii_grad is None:
            pos3d_radii_grad = pos3d_radii.new_zeros(pos3d_radii.shape)
        if conics_grad is None:
            conics_grad = pos3d_radii.new_zeros((ctx.num_gaussians, 6))
        grad_pos3d, grad_scale3d, grad_quat = _C.optim_to_render_backward(
            ctx.num_gaussians, pos3d, scale3d, quat, ctx.vol_size_voxel,
            ctx.vol_size_world, ctx.vol_center_pos, pos3d_radii_grad,
            conics_grad, pos3d_radii)
        return grad_pos3d, grad_scale3d, grad_quat, None, None, None, None, None
