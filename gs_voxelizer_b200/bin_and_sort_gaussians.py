"""Binning of Gaussians into 8x8x8 voxel tiles.

Drop-in for gs_voxelizer/bin_and_sort_gaussians.py:14-54 of the reference:
same name, arguments and outputs; not differentiable.
"""
from __future__ import annotations

from typing import Tuple

from torch import Tensor

from . import cuda as _C


def bin_and_sort_gaussians(
    num_gaussians: int,
    num_intersects: int,
    tile_min: Tensor,
    tile_max: Tensor,
    cum_tiles_hit: Tensor,
    vol_size: Tuple[int, int, int],
) -> Tuple[Tensor, Tensor]:
    """Map Gaussians to (tile, gaussian) intersections ordered by tile id,
    then by Gaussian id.

    Args:
        num_gaussians: number of Gaussians.
        num_intersects: total number of (tile, gaussian) intersections
            (``cum_tiles_hit[-1]``).
        tile_min, tile_max: [N,3] int32 tile boxes from optim_to_render.
        cum_tiles_hit: [N] int32 inclusive prefix sum of num_tiles_hit.
        vol_size: (depth, height, width) of the volume in voxels.

    Returns:
        gaussian_ids_sorted: [num_intersects] int32 Gaussian ids, grouped by
            tile.
        tile_bins: [T,2] int32 [start, end) of each tile's range; (0, 0) for
            tiles no Gaussian touches.
    """
    ids, bins = _C.bin_and_sort_gaussians(
        num_gaussians,
        num_intersects,
        tile_min.contiguous(),
        tile_max.contiguous(),
        cum_tiles_hit.contiguous(),
        vol_size,
    )
    return ids, bins
