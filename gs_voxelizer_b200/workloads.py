"""Seeded synthetic inputs for the benchmark configurations.

The reference publishes no dataset for this path; its benchmarks draw random
Gaussians and phantom volumes. These generators produce the distributions the
benchmark configurations name (see ``CONFIGS``): Gaussian parameters from a
numpy ``default_rng(seed)``, and a phantom target volume made of seeded random
ellipsoids, evaluated with torch on any device (so 2048^3 targets can be
built directly in HBM).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, Optional, Tuple

import numpy as np
import torch


@dataclass(frozen=True)
class Config:
    name: str
    vol: Tuple[int, int, int]              # (Z, Y, X) voxels
    n: int                                 # Gaussians
    pos: Tuple[float, float] = (0.0, 1.0)  # U[lo, hi]^3 (world units)
    scale: Tuple[float, float] = (0.005, 0.04)  # exp(U[ln lo, ln hi])
    intensity: Tuple[float, float] = (0.0, 1.0)
    channels: int = 1
    ellipsoids: int = 20
    world: Tuple[float, float, float] = (1.0, 1.0, 1.0)
    center: Tuple[float, float, float] = (0.5, 0.5, 0.5)
    seed: int = 0
    extra: Dict[str, float] = field(default_factory=dict)


def sweep_scale_hi(n: int) -> float:
    """Gaussian-count sweep: scale upper bound 0.02 * (1e5 / N)^(1/3)."""
    return 0.02 * (1e5 / n) ** (1.0 / 3.0)


CONFIGS = {
    # CPU-runnable case: 100x150x80, 5000 Gaussians, 20-ellipsoid phantom
    "cpu": Config("cpu", (100, 150, 80), 5000),
    # single-GPU training step: 256^3, 100k Gaussians, 64-ellipsoid phantom
    "step256": Config("step256", (256, 256, 256), 100_000, pos=(0.05, 0.95),
                      scale=(0.002, 0.02), intensity=(0.0, 0.5), ellipsoids=64),
    # z-slab sharded run: 2048^3, 8M Gaussians, 512-ellipsoid phantom
    "shard2048": Config("shard2048", (2048, 2048, 2048), 8_000_000,
                        pos=(0.0, 1.0), scale=(0.0005, 0.004),
                        intensity=(0.0, 0.5), ellipsoids=512),
}


def count_sweep(n: int) -> Config:
    return Config(f"sweepN{n}", (256, 256, 256), n, pos=(0.05, 0.95),
                  scale=(0.002, sweep_scale_hi(n)), intensity=(0.0, 0.5),
                  ellipsoids=64)


def volume_sweep(edge: int, channels: int) -> Config:
    return Config(f"vol{edge}c{channels}", (edge, edge, edge), 200_000,
                  pos=(0.05, 0.95), scale=(0.002, 0.02), intensity=(0.0, 0.5),
                  channels=channels, ellipsoids=64)


def gaussians(cfg: Config, seed: Optional[int] = None):
    """(pos3d [N,3], scale3d [N,3], quat [N,4], intensity [N,C]) float32."""
    rng = np.random.default_rng(cfg.seed if seed is None else seed)
    n = cfg.n
    pos = rng.uniform(cfg.pos[0], cfg.pos[1], size=(n, 3)).astype(np.float32)
    lo, hi = math.log(cfg.scale[0]), math.log(cfg.scale[1])
    scale = np.exp(rng.uniform(lo, hi, size=(n, 3))).astype(np.float32)
    q = rng.standard_normal(size=(n, 4))
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    quat = q.astype(np.float32)
    inten = rng.uniform(cfg.intensity[0], cfg.intensity[1],
                        size=(n, cfg.channels)).astype(np.float32)
    return pos, scale, quat, inten


def phantom(cfg: Config, device="cpu", seed: Optional[int] = None,
            z_range: Optional[Tuple[int, int]] = None) -> torch.Tensor:
    """Target volume [Z', Y, X, C] float32: sum of seeded random rotated
    ellipsoids of value U[0.2, 1] on a zero background, clipped to [0, 1].
    Channel c is scaled by a seeded U[0.5, 1] factor (1 for one channel).
    z_range restricts the output to voxel z in [z0, z1) (slab targets)."""
    rng = np.random.default_rng((cfg.seed if seed is None else seed) + 7919)
    Z, Y, X = cfg.vol
    z0, z1 = z_range if z_range is not None else (0, Z)
    K = cfg.ellipsoids
    centers = rng.uniform(0.0, 1.0, size=(K, 3)) * np.array([X, Y, Z])
    # semi-axes as a fraction of the smallest edge, shrinking as K grows
    frac = 0.18 * (20.0 / K) ** (1.0 / 3.0)
    axes = rng.uniform(0.3, 1.0, size=(K, 3)) * frac * min(X, Y, Z)
    axes = np.maximum(axes, 1.5)
    q = rng.standard_normal(size=(K, 4))
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    values = rng.uniform(0.2, 1.0, size=K)
    ch_scale = (np.ones(cfg.channels) if cfg.channels == 1
                else rng.uniform(0.5, 1.0, size=cfg.channels))

    vol = torch.zeros((z1 - z0, Y, X), dtype=torch.float32, device=device)
    for k in range(K):
        w, x, y, z = q[k]
        R = np.array([
            [1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y)],
            [2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x)],
            [2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)],
        ])
        r = axes[k].max()
        c = centers[k]
        lo = np.floor(c - r).astype(int)
        hi = np.ceil(c + r).astype(int) + 1
        xs = (max(lo[0], 0), min(hi[0], X))
        ys = (max(lo[1], 0), min(hi[1], Y))
        zs = (max(lo[2], z0), min(hi[2], z1))
        if xs[0] >= xs[1] or ys[0] >= ys[1] or zs[0] >= zs[1]:
            continue
        gz = torch.arange(zs[0], zs[1], device=device, dtype=torch.float32) + 0.5 - c[2]
        gy = torch.arange(ys[0], ys[1], device=device, dtype=torch.float32) + 0.5 - c[1]
        gx = torch.arange(xs[0], xs[1], device=device, dtype=torch.float32) + 0.5 - c[0]
        acc = None
        for i in range(3):  # body-frame coordinate i = sum_j R[j, i] * d_j
            u = (float(R[0, i]) * gx[None, None, :] + float(R[1, i]) * gy[None, :, None]
                 + float(R[2, i]) * gz[:, None, None]) / float(axes[k][i])
            acc = u * u if acc is None else acc + u * u
        mask = acc <= 1.0
        sub = vol[zs[0] - z0:zs[1] - z0, ys[0]:ys[1], xs[0]:xs[1]]
        sub.add_(mask.to(torch.float32) * float(values[k]))
        del acc, mask
    vol.clamp_(0.0, 1.0)
    out = vol.unsqueeze(-1)
    if cfg.channels > 1:
        out = out * torch.tensor(ch_scale, dtype=torch.float32, device=device)
    return out.contiguous()


def evaluations(tile_bins: torch.Tensor, vol: Tuple[int, int, int],
                tile_z: Optional[Tuple[int, int]] = None) -> int:
    """Gaussian-voxel evaluation count E = sum over tiles of
    (Gaussians in the tile) x (voxels of the tile inside the volume)."""
    Z, Y, X = vol
    tx, ty, tz = (X + 7) // 8, (Y + 7) // 8, (Z + 7) // 8
    tz0, tz1 = tile_z if tile_z is not None else (0, tz)
    b = tile_bins.to(torch.int64)
    n_t = (b[:, 1] - b[:, 0]).reshape(tz1 - tz0, ty, tx)
    dev = n_t.device
    wx = torch.clamp(X - 8 * torch.arange(tx, device=dev), max=8)
    wy = torch.clamp(Y - 8 * torch.arange(ty, device=dev), max=8)
    wz = torch.clamp(Z - 8 * torch.arange(tz0, tz1, device=dev), max=8)
    vox = wz[:, None, None] * wy[None, :, None] * wx[None, None, :]
    return int((n_t * vox).sum().item())
