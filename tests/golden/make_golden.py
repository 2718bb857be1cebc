"""Generate the golden fixtures of tests/golden/ from the reference's own
CUDA extension (oracle/_ref, built from the reference's unmodified sources).

Needs a GPU and the built reference; run on the GPU box:
    python tests/golden/make_golden.py OUT_DIR
Each case stores the seeded inputs and the reference's outputs of
projection, binning, forward and per-Gaussian backward and projection
backward. dL/dvol is not stored: it is standard normal from
numpy default_rng(100 + seed), drawn before the projection-backward inputs. The CPU test test_golden_cpu.py checks the
oracle against them.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from gs_voxelizer_b200.workloads import Config, gaussians  # noqa: E402
from oracle import ref_api  # noqa: E402

CASES = {
    "cfg1_cpu_c1": Config("golden", (100, 150, 80), 5000, seed=0),
    "small_c2": Config("golden", (24, 33, 41), 600, scale=(0.01, 0.06),
                       channels=2, seed=1, world=(0.8, 1.0, 1.2),
                       center=(0.4, 0.5, 0.6)),
    "small_c4": Config("golden", (20, 20, 20), 300, scale=(0.02, 0.1),
                       channels=4, seed=2),
}


def main(out_dir):
    ext = ref_api.ext()
    os.makedirs(out_dir, exist_ok=True)
    for name, cfg in CASES.items():
        pos, scale, quat, inten = gaussians(cfg)
        d = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
        P, S, Q, I = d(pos), d(scale), d(quat), d(inten)
        pr, cq, tmin, tmax, nt = ext.optim_to_render_forward(
            cfg.n, P, S, Q, I, cfg.vol, cfg.world, cfg.center)
        cum = torch.cumsum(nt, 0, dtype=torch.int32)
        n_isect = int(cum[-1].item())
        ids, bins = ext.bin_and_sort_gaussians(cfg.n, n_isect, tmin, tmax, cum, cfg.vol)
        vol = ext.voxelize_forward(cfg.vol, ids, bins, pr, cq, I)
        rng = np.random.default_rng(100 + cfg.seed)
        W = rng.standard_normal(tuple(vol.shape)).astype(np.float32)
        gp, gc, gi = ext.voxelize_backward_per_gaussian(cfg.vol, ids, bins, pr,
                                                        cq, I, d(W))
        Gp = rng.standard_normal((cfg.n, 4)).astype(np.float32)
        Gc = rng.standard_normal((cfg.n, 6)).astype(np.float32)
        dp, ds, dq = ext.optim_to_render_backward(cfg.n, P, S, Q, cfg.vol,
                                                  cfg.world, cfg.center,
                                                  d(Gp), d(Gc), pr)
        h = lambda t: t.detach().cpu().numpy()  # noqa: E731
        v = h(vol)
        # large volumes keep four z-slices plus per-slice sums (fixture size)
        zs = (np.arange(v.shape[0]) if v.size <= 200_000
              else np.array([0, v.shape[0] // 3, v.shape[0] // 2, v.shape[0] - 1]))
        np.savez_compressed(
            os.path.join(out_dir, f"{name}.npz"),
            vol_size=np.array(cfg.vol), world=np.array(cfg.world, np.float32),
            center=np.array(cfg.center, np.float32),
            pos3d=pos, scale3d=scale, quat=quat, intensities=inten,
            pos3d_radii=h(pr), conics=h(cq), tile_min=h(tmin), tile_max=h(tmax),
            num_tiles_hit=h(nt), gaussian_ids_sorted=h(ids), tile_bins=h(bins),
            volume_z=zs, volume_slices=v[zs],
            volume_z_sums=v.astype(np.float64).sum(axis=(1, 2, 3)),
            pos_grad=h(gp), conic_grad=h(gc),
            intensity_grad=h(gi), pos3d_radii_grad_in=Gp, conics_grad_in=Gc,
            pos3d_grad=h(dp), scale3d_grad=h(ds), quat_grad=h(dq))
        print(name, "isect", n_isect, "max vol", float(vol.max()))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.dirname(os.path.abspath(__file__)))
