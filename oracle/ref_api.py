"""The reference's Python API flow on top of its own compiled extension
(oracle/_ref, built by oracle/build_ref.py from the reference's unmodified
CUDA sources).

TEST / BENCH INFRASTRUCTURE ONLY: used by the reference-parity tests and by
``bench.py --impl reference``. It restates, call for call, the autograd glue
of the reference's gs_voxelizer/optim_to_render.py:53-149 and
gs_voxelizer/voxelize.py:52-173 (cumsum + host sync, bin_and_sort, forward,
per-Gaussian or per-voxel backward, projection backward), because those
Python files cannot travel to the GPU box. Every kernel on this path is the
reference's own.
"""
from __future__ import annotations

import torch
from torch.autograd import Function

from oracle import build_ref

_ext = None


def ext():
    global _ext
    if _ext is None:
        _ext = build_ref.load_reference()
        if _ext is None:
            raise ImportError("reference extension not built (oracle/_ref)")
    return _ext


def available() -> bool:
    return build_ref.built_library() is not None


class _RefOptimToRender(Function):
    @staticmethod
    def forward(ctx, pos3d, scale3d, quat, intensities, vol, world, center):
        n = pos3d.size(-2)
        out = ext().optim_to_render_forward(n, pos3d, scale3d, quat,
                                            intensities, vol, world, center)
        ctx.args = (n, vol, world, center)
        ctx.save_for_backward(pos3d, scale3d, quat, out[0])
        ctx.mark_non_differentiable(out[2], out[3], out[4])
        return out

    @staticmethod
    def backward(ctx, g_pos, g_conic, *_):
        pos3d, scale3d, quat, pos_radii = ctx.saved_tensors
        n, vol, world, center = ctx.args
        if g_pos is None:
            g_pos = torch.zeros_like(pos_radii)
        if g_conic is None:
            g_conic = pos_radii.new_zeros((n, 6))
        gp, gs, gq = ext().optim_to_render_backward(
            n, pos3d, scale3d, quat, vol, world, center, g_pos.contiguous(),
            g_conic.contiguous(), pos_radii)
        return gp, gs, gq, None, None, None, None


class _RefVoxelize(Function):
    @staticmethod
    def forward(ctx, pos_radii, conics, intensities, vol, tile_min, tile_max,
                num_tiles_hit, per_gaussian):
        if intensities.dim() == 1:
            intensities = intensities.unsqueeze(-1)
        n = pos_radii.size(-2)
        ctx.vol, ctx.per_gaussian = vol, per_gaussian
        cum = torch.cumsum(num_tiles_hit, dim=0, dtype=torch.int32)
        n_isect = int(cum[-1].item()) if n else 0
        ctx.n_isect = n_isect
        if n_isect < 1:
            out = torch.zeros(*vol, intensities.shape[-1], device=pos_radii.device)
            ids = torch.zeros(0, 1, device=pos_radii.device, dtype=torch.int32)
            bins = torch.zeros(0, 3, device=pos_radii.device, dtype=torch.int32)
        else:
            ids, bins = ext().bin_and_sort_gaussians(
                n, n_isect, tile_min.contiguous(), tile_max.contiguous(),
                cum.contiguous(), vol)
            out = ext().voxelize_forward(vol, ids, bins, pos_radii, conics,
                                         intensities)
        ctx.save_for_backward(pos_radii, conics, intensities, ids, bins)
        return out

    @staticmethod
    def backward(ctx, g):
        pos_radii, conics, intensities, ids, bins = ctx.saved_tensors
        if ctx.n_isect < 1:
            return (torch.zeros_like(pos_radii), torch.zeros_like(conics),
                    torch.zeros_like(intensities), None, None, None, None, None)
        fn = (ext().voxelize_backward_per_gaussian if ctx.per_gaussian
              else ext().voxelize_backward)
        gp, gc, gi = fn(ctx.vol, ids, bins, pos_radii, conics, intensities,
                        g.contiguous())
        return gp, gc, gi, None, None, None, None, None


def optim_to_render(pos3d, scale3d, quat, intensities, vol, world, center):
    return _RefOptimToRender.apply(pos3d.contiguous(), scale3d.contiguous(),
                                   quat.contiguous(), intensities.contiguous(),
                                   tuple(vol), tuple(world), tuple(center))


def voxelize_gaussians(pos_radii, conics, intensities, vol, tile_min, tile_max,
                       num_tiles_hit, use_per_gaussian_backward=True):
    return _RefVoxelize.apply(pos_radii.contiguous(), conics.contiguous(),
                              intensities.contiguous(), tuple(vol), tile_min,
                              tile_max, num_tiles_hit,
                              use_per_gaussian_backward)
