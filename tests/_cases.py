"""Shared test inputs and float64 numpy restatements used as independent
cross-checks of the C oracle (oracle/gsv_oracle.c)."""
from __future__ import annotations

import numpy as np

from gs_voxelizer_b200.workloads import Config, gaussians


def small_config(vol=(40, 48, 56), n=300, seed=0, channels=1,
                 scale=(0.01, 0.05), pos=(0.0, 1.0), intensity=(0.0, 1.0),
                 world=(1.0, 1.0, 1.0), center=(0.5, 0.5, 0.5)) -> Config:
    return Config("test", tuple(vol), n, pos=pos, scale=scale,
                  intensity=intensity, channels=channels, ellipsoids=5,
                  world=tuple(world), center=tuple(center), seed=seed)


def inputs(cfg: Config):
    return gaussians(cfg)


def rotation64(q):
    """Rotation (math convention, row-major) of the quaternion slots
    (w, x, y, z) after normalisation; equals the reference's column-major
    GLM matrix read as R_math[r][c] = m[c][r]."""
    q = np.asarray(q, np.float64)
    q = q / np.linalg.norm(q, axis=-1, keepdims=True)
    w, x, y, z = q[..., 0], q[..., 1], q[..., 2], q[..., 3]
    # GLM columns: col0 = (1-2(yy+zz), 2(xy-wz), 2(xz+wy)), ...
    m = np.empty(q.shape[:-1] + (3, 3))
    cols = [
        (1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y)),
        (2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x)),
        (2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)),
    ]
    for c in range(3):
        for r in range(3):
            m[..., r, c] = cols[c][r]
    return m


def voxel_cov64(scale, quat, vol, world):
    """Voxel-space covariance (S R)^T (S R) with S = diag(scale), scaled by
    diag(1/voxel size) on both sides (optim_to_render.cu:84-103)."""
    Z, Y, X = vol
    vox = np.array([world[2] / X, world[1] / Y, world[0] / Z])
    R = rotation64(quat)
    S = np.asarray(scale, np.float64)[..., :, None] * np.eye(3)
    M = S @ R
    cov = np.swapaxes(M, -1, -2) @ M
    D = np.eye(3) / vox
    return D @ cov @ D


def conic_from_cov(cov):
    Q = np.linalg.inv(cov)
    return np.stack([Q[..., 0, 0], Q[..., 0, 1], Q[..., 0, 2], Q[..., 1, 1],
                     Q[..., 1, 2], Q[..., 2, 2]], axis=-1)


def pixel_pos64(pos, vol, world, center):
    Z, Y, X = vol
    vox = np.array([world[2] / X, world[1] / Y, world[0] / Z])
    c = np.array([center[2], center[1], center[0]])
    w = np.array([world[2], world[1], world[0]])
    return (np.asarray(pos, np.float64) - c + 0.5 * w) / vox


def sigma64(q, d):
    """-1/2 d^T Q d with the reference's conic layout (voxelize.cu:125-131)."""
    a, b, c, dd, e, f = (q[..., k] for k in range(6))
    dx, dy, dz = d[..., 0], d[..., 1], d[..., 2]
    return -0.5 * (a * dx * dx + dd * dy * dy + f * dz * dz) - (
        b * dx * dy + c * dx * dz + e * dy * dz)


def stable_binning(tile_min, tile_max, vol):
    """Keys emitted per Gaussian in z, y, x order, then a stable argsort:
    the reference's map_gaussian_to_intersects + CUB stable radix sort."""
    Z, Y, X = vol
    tx, ty, tz = (X + 7) // 8, (Y + 7) // 8, (Z + 7) // 8
    keys, gids = [], []
    for g in range(tile_min.shape[0]):
        for k in range(tile_min[g, 2], tile_max[g, 2]):
            for j in range(tile_min[g, 1], tile_max[g, 1]):
                for i in range(tile_min[g, 0], tile_max[g, 0]):
                    keys.append(k * ty * tx + j * tx + i)
                    gids.append(g)
    keys = np.asarray(keys, np.int64)
    gids = np.asarray(gids, np.int32)
    order = np.argsort(keys, kind="stable")
    ks, ids = keys[order], gids[order]
    bins = np.zeros((tx * ty * tz, 2), np.int32)
    for idx in range(len(ks)):
        t = ks[idx]
        if idx == 0 or ks[idx - 1] != t:
            bins[t, 0] = idx
        if idx == len(ks) - 1 or ks[idx + 1] != t:
            bins[t, 1] = idx + 1
    return ids, bins


def forward64(vol, ids, bins, pos_radii, conics, intens):
    """Direct float64 evaluation of the forward sum with the two culls."""
    Z, Y, X = vol
    intens = np.asarray(intens, np.float64)
    if intens.ndim == 1:
        intens = intens[:, None]
    C = intens.shape[1]
    tx, ty = (X + 7) // 8, (Y + 7) // 8
    out = np.zeros((Z, Y, X, C))
    lz, ly, lx = np.meshgrid(np.arange(8), np.arange(8), np.arange(8), indexing="ij")
    for t in range(bins.shape[0]):
        b0, b1 = bins[t]
        if b1 <= b0:
            continue
        ox, oy, oz = 8 * (t % tx), 8 * ((t // tx) % ty), 8 * (t // (tx * ty))
        x, y, z = ox + lx, oy + ly, oz + lz
        inside = (x < X) & (y < Y) & (z < Z)
        vx, vy, vz = x + 0.5, y + 0.5, z + 0.5
        acc = np.zeros((8, 8, 8, C))
        for k in range(b0, b1):
            g = ids[k]
            p = pos_radii[g].astype(np.float64)
            d = np.stack([p[0] - vx, p[1] - vy, p[2] - vz], axis=-1)
            s = sigma64(conics[g].astype(np.float64), d)
            alpha = np.exp(np.minimum(s, 0.0))
            ok = (s <= 0) & np.isfinite(s) & (alpha * intens[g].mean() >= 1e-6)
            acc += np.where(ok[..., None], alpha[..., None] * intens[g], 0.0)
        zz, yy, xx = z[inside], y[inside], x[inside]
        out[zz, yy, xx] = acc[inside]
    return out
