"""numpy front end of the CPU oracle (oracle/gsv_oracle.c).

TEST INFRASTRUCTURE ONLY. The parity tests, ``__graft_entry__.smoke()`` and
bench.py's ``cpu_baseline`` leg use these functions as the checker; the
product package ``gs_voxelizer_b200`` never imports this module.

The functions mirror the reference's extension entry points
(gs_voxelizer/cuda/bindings.cu of PaPieta/gs-voxelizer) on numpy arrays:
inputs are float32 / int32 C-contiguous arrays, tuples are (z, y, x).
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_lib = None


def lib():
    global _lib
    if _lib is None:
        from oracle import build as _build  # noqa: WPS433

        path = _build.build()
        L = ctypes.CDLL(str(path))
        P = ctypes.c_void_p
        i32, i64, f64 = ctypes.c_int, ctypes.c_int64, ctypes.c_double
        L.oracle_project_fwd.argtypes = [i32, i32] + [P] * 13
        L.oracle_project_fwd.restype = None
        L.oracle_project_bwd.argtypes = [i32] + [P] * 11
        L.oracle_project_bwd.restype = None
        L.oracle_bin.argtypes = [i32, P, P, P, i32, i32, P, P, i64]
        L.oracle_bin.restype = i64
        L.oracle_vox_fwd.argtypes = [P, i32, i32, i32, P, P, P, P, P, P]
        L.oracle_vox_fwd.restype = None
        L.oracle_vox_bwd.argtypes = [P, i32, i32, i32, i32] + [P] * 9
        L.oracle_vox_bwd.restype = None
        L.oracle_l1.argtypes = [i64, P, P, f64, P]
        L.oracle_l1.restype = f64
        L.oracle_ssim3d.argtypes = [i32, i32, i32, i32, P, P, f64, f64, P, i32, P]
        L.oracle_ssim3d.restype = f64
        L.oracle_tv3d.argtypes = [i32, i32, i32, i32, P, i32, f64, P]
        L.oracle_tv3d.restype = f64
        L.oracle_num_threads.argtypes = []
        L.oracle_num_threads.restype = i32
        _lib = L
    return _lib


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _i32(a):
    return np.ascontiguousarray(a, dtype=np.int32)


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p) if a is not None else None


def num_threads() -> int:
    return int(lib().oracle_num_threads())


def optim_to_render_forward(pos3d, scale3d, quat, intensities, vol_size_voxel,
                            vol_size_world, vol_center_pos, return_bounds=False):
    """optim_to_render.cu:48-172. Returns (pos3d_radii, conics, tile_min,
    tile_max, num_tiles_hit[, bounds]) where bounds [N,6] holds the
    pre-truncation tile values used to flag boundary-ambiguous integers."""
    pos3d, scale3d, quat = _f32(pos3d), _f32(scale3d), _f32(quat)
    intens = _f32(intensities)
    n = pos3d.shape[0]
    C = 1 if intens.ndim == 1 else intens.shape[1]
    vol = _i32(vol_size_voxel)
    world = _f32(vol_size_world)
    center = _f32(vol_center_pos)
    pr = np.zeros((n, 4), np.float32)
    cq = np.zeros((n, 6), np.float32)
    tmin = np.zeros((n, 3), np.int32)
    tmax = np.zeros((n, 3), np.int32)
    nt = np.zeros((n,), np.int32)
    bounds = np.zeros((n, 6), np.float32)
    lib().oracle_project_fwd(n, C, _p(pos3d), _p(scale3d), _p(quat),
                             _p(intens), _p(vol), _p(world), _p(center),
                             _p(pr), _p(cq), _p(tmin), _p(tmax), _p(nt),
                             _p(bounds))
    if return_bounds:
        return pr, cq, tmin, tmax, nt, bounds
    return pr, cq, tmin, tmax, nt


def optim_to_render_backward(pos3d, scale3d, quat, vol_size_voxel,
                             vol_size_world, pos3d_radii_grad, conics_grad,
                             pos3d_radii):
    """optim_to_render.cu:246-336 -> (pos3d_grad, scale3d_grad, quat_grad)."""
    pos3d, scale3d, quat = _f32(pos3d), _f32(scale3d), _f32(quat)
    n = pos3d.shape[0]
    vol = _i32(vol_size_voxel)
    world = _f32(vol_size_world)
    gpr, gc, pr = _f32(pos3d_radii_grad), _f32(conics_grad), _f32(pos3d_radii)
    gp = np.zeros((n, 3), np.float32)
    gs = np.zeros((n, 3), np.float32)
    gq = np.zeros((n, 4), np.float32)
    lib().oracle_project_bwd(n, _p(pos3d), _p(scale3d), _p(quat), _p(vol),
                             _p(world), _p(gpr), _p(gc), _p(pr), _p(gp),
                             _p(gs), _p(gq))
    return gp, gs, gq


def num_tiles(vol_size_voxel, tile_z=None):
    Z, Y, X = (int(v) for v in vol_size_voxel)
    tz0, tz1 = tile_z if tile_z is not None else (0, (Z + 7) // 8)
    return (tz1 - tz0) * ((Y + 7) // 8) * ((X + 7) // 8)


def bin_and_sort_gaussians(tile_min, tile_max, vol_size_voxel, tile_z=None):
    """bin_and_sort_gaussians.cu:11-62 + the stable sort of bindings.cu:316.
    Returns (gaussian_ids_sorted [I], tile_bins [T,2])."""
    tmin, tmax = _i32(tile_min), _i32(tile_max)
    vol = _i32(vol_size_voxel)
    tz0, tz1 = tile_z if tile_z is not None else (0, -1)
    T = num_tiles(vol_size_voxel, tile_z)
    bins = np.zeros((T, 2), np.int32)
    n = tmin.shape[0]
    total = lib().oracle_bin(n, _p(tmin), _p(tmax), _p(vol), tz0, tz1, None,
                             _p(bins), 0)
    ids = np.zeros((total,), np.int32)
    got = lib().oracle_bin(n, _p(tmin), _p(tmax), _p(vol), tz0, tz1, _p(ids),
                           _p(bins), total)
    assert got == total
    return ids, bins


def voxelize_forward(vol_size_voxel, ids, tile_bins, pos3d_radii, conics,
                     intensities, tile_z=None):
    """voxelize.cu:39-164 -> volume [Z', Y, X, C]."""
    Z, Y, X = (int(v) for v in vol_size_voxel)
    intens = _f32(intensities)
    C = 1 if intens.ndim == 1 else intens.shape[1]
    tz0, tz1 = tile_z if tile_z is not None else (0, -1)
    zb = tz0 * 8
    ze = Z if tz1 < 0 else min(Z, tz1 * 8)
    out = np.zeros((ze - zb, Y, X, C), np.float32)
    vol = _i32(vol_size_voxel)
    ids, bins = _i32(ids), _i32(tile_bins)
    pr, cq = _f32(pos3d_radii), _f32(conics)
    lib().oracle_vox_fwd(_p(vol), tz0, tz1, C, _p(ids), _p(bins), _p(pr),
                         _p(cq), _p(intens), _p(out))
    return out


def voxelize_backward(vol_size_voxel, tile_min, tile_max, pos3d_radii, conics,
                      intensities, vol_grad, tile_z=None):
    """voxelize.cu:368-574 -> (pos3d_grad [N,4], conics_grad [N,6],
    intensities_grad [N,C])."""
    intens = _f32(intensities)
    if intens.ndim == 1:
        intens = intens[:, None]
    C = intens.shape[1]
    n = intens.shape[0]
    tz0, tz1 = tile_z if tile_z is not None else (0, -1)
    vol = _i32(vol_size_voxel)
    tmin, tmax = _i32(tile_min), _i32(tile_max)
    pr, cq, g = _f32(pos3d_radii), _f32(conics), _f32(vol_grad)
    gp = np.zeros((n, 4), np.float32)
    gc = np.zeros((n, 6), np.float32)
    gi = np.zeros((n, C), np.float32)
    lib().oracle_vox_bwd(_p(vol), tz0, tz1, C, n, _p(tmin), _p(tmax), _p(pr),
                         _p(cq), _p(intens), _p(g), _p(gp), _p(gc), _p(gi))
    return gp, gc, gi


def l1_loss_and_grad(vol, target):
    """mean |vol - target| and its gradient sign(vol - target) / numel."""
    v, t = _f32(vol), _f32(target)
    g = np.empty_like(v)
    loss = lib().oracle_l1(v.size, _p(v), _p(t), float(v.size), _p(g))
    return loss, g


def ssim_window(sigma: float = 1.5, radius: int = 5) -> np.ndarray:
    """Normalised 1-D Gaussian window of 2 * radius + 1 taps (float64)."""
    k = np.arange(-radius, radius + 1, dtype=np.float64)
    w = np.exp(-k * k / (2.0 * sigma * sigma))
    return w / w.sum()


def ssim3d(img1, img2, c1=0.01 ** 2, c2=0.03 ** 2, grad=True):
    """Mean 3D SSIM of planar volumes [..., D, H, W] (leading dims are
    channels) and, with grad, d SSIM / d img1 (float32, same shape)."""
    a, b = _f32(img1), _f32(img2)
    D, H, W = a.shape[-3:]
    nch = int(np.prod(a.shape[:-3])) if a.ndim > 3 else 1
    w = np.ascontiguousarray(ssim_window(), dtype=np.float64)
    g = np.empty_like(a) if grad else None
    v = lib().oracle_ssim3d(nch, D, H, W, _p(a), _p(b), c1, c2, _p(w), 5, _p(g))
    return (v, g) if grad else v


def tv3d(vol, isotropic=True, eps=1e-8, grad=True):
    """3D total variation (mean over voxels and channels) of planar volumes
    [..., D, H, W] and, with grad, its gradient."""
    x = _f32(vol)
    D, H, W = x.shape[-3:]
    nch = int(np.prod(x.shape[:-3])) if x.ndim > 3 else 1
    g = np.empty_like(x) if grad else None
    v = lib().oracle_tv3d(nch, D, H, W, _p(x), 1 if isotropic else 0, eps, _p(g))
    return (v, g) if grad else v
