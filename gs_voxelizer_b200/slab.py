"""z-slab sharding of the voxelization across GPUs (one process per GPU).

The reference is single-GPU. Here the volume's tile layers are split into
contiguous z-slabs, one per rank:

  1. every rank projects all Gaussians (cheap, replicated);
  2. each rank bins only the (tile, Gaussian) pairs whose tile lies in its
     slab (``gsv_bin_and_sort_gaussians_slab``; the result equals the
     full-volume binning restricted to the slab);
  3. each rank voxelizes its slab and computes its part of the loss, with the
     loss normalised by the GLOBAL voxel count so slab losses sum to the
     full-volume loss;
  4. the per-Gaussian gradients (position, conic, intensity) of all slabs are
     summed with ONE all-reduce (NCCL over NVLink on GPUs, gloo on CPU);
  5. every rank runs the projection backward on the summed gradients, so all
     ranks hold identical parameter gradients.

No data-path collective is needed in the forward pass.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.distributed as dist
from torch.autograd import Function

from . import cuda as _C
from ._lib import check, i3, lib

TILE = 8


def tile_layers(vol_size: Tuple[int, int, int]) -> int:
    return (int(vol_size[0]) + TILE - 1) // TILE


def slab_bounds(vol_size: Tuple[int, int, int], world_size: int,
                rank: int) -> Tuple[int, int]:
    """Contiguous, balanced split of the tile layers: rank r gets
    [tz0, tz1) with sizes differing by at most one layer."""
    Tz = tile_layers(vol_size)
    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError(f"bad rank {rank} of {world_size}")
    base, extra = divmod(Tz, world_size)
    tz0 = rank * base + min(rank, extra)
    tz1 = tz0 + base + (1 if rank < extra else 0)
    return tz0, tz1


class SlabPlan:
    """Binning / voxelization of the tile layers [tz0, tz1) of a volume."""

    def __init__(self, vol_size: Tuple[int, int, int], tz0: int, tz1: int):
        self.vol = tuple(int(v) for v in vol_size)
        Tz = tile_layers(self.vol)
        if not 0 <= tz0 <= tz1 <= Tz:
            raise ValueError(f"tile z range [{tz0}, {tz1}) outside [0, {Tz})")
        self.tz0, self.tz1 = int(tz0), int(tz1)
        self.z_begin = self.tz0 * TILE
        self.z_end = min(self.vol[0], self.tz1 * TILE)
        ty = (self.vol[1] + TILE - 1) // TILE
        tx = (self.vol[2] + TILE - 1) // TILE
        self.num_tiles = (self.tz1 - self.tz0) * ty * tx

    @property
    def shape(self) -> Tuple[int, int, int]:
        return (self.z_end - self.z_begin, self.vol[1], self.vol[2])

    def count(self, tile_min: torch.Tensor, tile_max: torch.Tensor) -> int:
        n = int(tile_min.shape[0])
        out = torch.empty((1,), dtype=torch.int64, device=tile_min.device)
        check(lib.gsv_count_slab_intersects(
            n, tile_min.data_ptr(), tile_max.data_ptr(), self.tz0, self.tz1,
            out.data_ptr(), _C._stream(tile_min.device)))
        return int(out.item())

    def bin(self, tile_min: torch.Tensor, tile_max: torch.Tensor,
            num_intersects: Optional[int] = None):
        tile_min, tile_max = tile_min.contiguous(), tile_max.contiguous()
        n = int(tile_min.shape[0])
        if num_intersects is None:
            num_intersects = self.count(tile_min, tile_max)
        dev = tile_min.device
        ids = torch.empty((num_intersects,), dtype=torch.int32, device=dev)
        bins = torch.empty((self.num_tiles, 2), dtype=torch.int32, device=dev)
        v = i3(self.vol)
        ws = _C._workspace(lib.gsv_bin_and_sort_slab_workspace_bytes(
            n, num_intersects, v, self.tz0, self.tz1), dev)
        check(lib.gsv_bin_and_sort_gaussians_slab(
            n, num_intersects, tile_min.data_ptr(), tile_max.data_ptr(), v,
            self.tz0, self.tz1, _C._ptr(ids), _C._ptr(bins), ws.data_ptr(),
            ws.numel(), _C._stream(dev)))
        return ids, bins

    def _ws(self, n, C, n_isect, dev):
        return _C._workspace(lib.gsv_voxelize_slab_workspace_bytes(
            n, C, n_isect, i3(self.vol), self.tz0, self.tz1), dev)

    def forward(self, ids, bins, pos3d_radii, conics, intensities):
        C = _C._vox_inputs(ids, bins, pos3d_radii, conics, intensities)
        n, n_isect, dev = int(pos3d_radii.shape[0]), int(ids.numel()), pos3d_radii.device
        out = torch.empty((*self.shape, C), dtype=torch.float32, device=dev)
        ws = self._ws(n, C, n_isect, dev)
        check(lib.gsv_voxelize_forward_slab(
            i3(self.vol), self.tz0, self.tz1, C, n, n_isect, _C._ptr(ids),
            _C._ptr(bins), _C._ptr(pos3d_radii), _C._ptr(conics),
            _C._ptr(intensities), _C._ptr(out), ws.data_ptr(), ws.numel(),
            _C._stream(dev)))
        return out

    def backward(self, ids, bins, pos3d_radii, conics, intensities, vol_grad):
        C = _C._vox_inputs(ids, bins, pos3d_radii, conics, intensities)
        vol_grad = vol_grad.contiguous()
        n, n_isect, dev = int(pos3d_radii.shape[0]), int(ids.numel()), pos3d_radii.device
        f = dict(device=dev, dtype=torch.float32)
        gp = torch.empty((n, 4), **f)
        gc = torch.empty((n, 6), **f)
        gi = torch.empty((n, C), **f)
        ws = self._ws(n, C, n_isect, dev)
        check(lib.gsv_voxelize_backward_per_gaussian_slab(
            i3(self.vol), self.tz0, self.tz1, C, n, n_isect, _C._ptr(ids),
            _C._ptr(bins), _C._ptr(pos3d_radii), _C._ptr(conics),
            _C._ptr(intensities), _C._ptr(vol_grad), _C._ptr(gp), _C._ptr(gc),
            _C._ptr(gi), ws.data_ptr(), ws.numel(), _C._stream(dev)))
        return gp, gc, gi


def allreduce_gaussian_grads(grads, group=None):
    """Sum the per-Gaussian gradient tensors over the process group with a
    single all-reduce of one flat buffer."""
    if not (dist.is_available() and dist.is_initialized()):
        return grads
    if dist.get_world_size(group) == 1:
        return grads
    flat = torch.cat([g.reshape(-1) for g in grads])
    dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
    out, off = [], 0
    for g in grads:
        out.append(flat[off:off + g.numel()].view_as(g))
        off += g.numel()
    return out


class _SlabVoxelize(Function):
    @staticmethod
    def forward(ctx, pos3d_radii, conics, intensities, plan, tile_min,
                tile_max, group):
        one_d = intensities.dim() == 1
        if one_d:
            intensities = intensities.unsqueeze(-1)
        ids, bins = plan.bin(tile_min, tile_max)
        out = plan.forward(ids, bins, pos3d_radii, conics, intensities)
        ctx.plan, ctx.group, ctx.one_d = plan, group, one_d
        ctx.save_for_backward(pos3d_radii, conics, intensities, ids, bins)
        return out

    @staticmethod
    def backward(ctx, grad):
        pr, cq, inten, ids, bins = ctx.saved_tensors
        gp, gc, gi = ctx.plan.backward(ids, bins, pr, cq, inten, grad)
        gp, gc, gi = allreduce_gaussian_grads([gp, gc, gi], ctx.group)
        if ctx.one_d:
            gi = gi.reshape(-1)
        return gp, gc, gi, None, None, None, None


def voxelize_gaussians_slab(pos3d_radii, conics, intensities, plan: SlabPlan,
                            tile_min, tile_max, group=None) -> torch.Tensor:
    """Differentiable voxelization of one z-slab. The backward all-reduces
    the per-Gaussian gradients over ``group`` (when torch.distributed is
    initialised), so the projection backward that follows sees the gradient
    of the whole volume on every rank."""
    return _SlabVoxelize.apply(pos3d_radii.contiguous(), conics.contiguous(),
                               intensities.contiguous(), plan,
                               tile_min.contiguous(), tile_max.contiguous(),
                               group)
