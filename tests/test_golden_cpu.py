"""The CPU oracle against golden outputs of the reference's own CUDA
extension (tests/golden/*.npz, written by tests/golden/make_golden.py on a
B200 from the reference's unmodified sources). This pins the oracle that the
GPU parity tests rely on. No GPU needed.

The reference runs with --use_fast_math (approximate divide / sqrt / log /
exp, fused multiply-adds); the oracle evaluates in IEEE float, so
  * tile bounds must match except where the pre-truncation value lies within
    1e-5 (relative) of an integer (counted; must be rare),
  * binning (integers from the same tile boxes) must match exactly,
  * floats within the tolerances of the GPU parity tests.
"""
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O

GOLDEN = sorted((Path(__file__).parent / "golden").glob("*.npz"))


def _load(path):
    with np.load(path) as z:
        return {k: z[k] for k in z.files}


def _grad_close(got, want, name):
    want = want.astype(np.float64)
    err = np.abs(got.astype(np.float64) - want)
    tol = 1e-4 * np.abs(want) + 1e-4 * max(np.abs(want).max(), 1e-30)
    assert (err <= tol).all(), f"{name}: {(err > tol).sum()} out of tolerance"


def test_golden_fixtures_present():
    assert len(GOLDEN) >= 3


@pytest.mark.parametrize("path", GOLDEN, ids=lambda p: p.stem)
def test_oracle_projection_against_reference(path):
    g = _load(path)
    pr, cq, tmin, tmax, nt, bounds = O.optim_to_render_forward(
        g["pos3d"], g["scale3d"], g["quat"], g["intensities"], g["vol_size"],
        g["world"], g["center"], return_bounds=True)
    same = (tmin == g["tile_min"]).all(1) & (tmax == g["tile_max"]).all(1) & (nt == g["num_tiles_hit"])
    frac = np.abs(bounds - np.round(bounds))
    ambiguous = (frac < 1e-5 * np.maximum(1.0, np.abs(bounds))).any(1)
    assert (same | ambiguous).all()
    assert (~same).sum() <= max(2, len(nt) // 1000)
    ok = same & (nt > 0)
    np.testing.assert_allclose(pr[ok], g["pos3d_radii"][ok], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(cq[ok], g["conics"][ok], rtol=2e-3,
                               atol=2e-5 * np.abs(g["conics"]).max())


@pytest.mark.parametrize("path", GOLDEN, ids=lambda p: p.stem)
def test_oracle_binning_against_reference(path):
    g = _load(path)
    ids, bins = O.bin_and_sort_gaussians(g["tile_min"], g["tile_max"], g["vol_size"])
    np.testing.assert_array_equal(ids, g["gaussian_ids_sorted"])
    np.testing.assert_array_equal(bins, g["tile_bins"])


@pytest.mark.parametrize("path", GOLDEN, ids=lambda p: p.stem)
def test_oracle_voxelize_against_reference(path):
    g = _load(path)
    vol = O.voxelize_forward(g["vol_size"], g["gaussian_ids_sorted"], g["tile_bins"],
                             g["pos3d_radii"], g["conics"], g["intensities"])
    got = vol[g["volume_z"]].astype(np.float64)
    want = g["volume_slices"].astype(np.float64)
    assert (np.abs(got - want) <= 1e-5 * np.abs(want) + 1e-6).all()
    np.testing.assert_allclose(vol.astype(np.float64).sum(axis=(1, 2, 3)),
                               g["volume_z_sums"], rtol=1e-5, atol=1e-4)
    seed = {"cfg1_cpu_c1": 0, "small_c2": 1, "small_c4": 2}[path.stem]
    rng = np.random.default_rng(100 + seed)
    W = rng.standard_normal(vol.shape).astype(np.float32)
    gp, gc, gi = O.voxelize_backward(g["vol_size"], g["tile_min"], g["tile_max"],
                                     g["pos3d_radii"], g["conics"], g["intensities"], W)
    _grad_close(gp, g["pos_grad"], "pos")
    _grad_close(gc, g["conic_grad"], "conic")
    _grad_close(gi, g["intensity_grad"], "intensity")
    Gp = rng.standard_normal((len(gp), 4)).astype(np.float32)
    Gc = rng.standard_normal((len(gp), 6)).astype(np.float32)
    np.testing.assert_array_equal(Gp, g["pos3d_radii_grad_in"])
    dp, ds, dq = O.optim_to_render_backward(g["pos3d"], g["scale3d"], g["quat"],
                                            g["vol_size"], g["world"], Gp, Gc,
                                            g["pos3d_radii"])
    _grad_close(dp, g["pos3d_grad"], "pos3d")
    _grad_close(ds, g["scale3d_grad"], "scale3d")
    _grad_close(dq, g["quat_grad"], "quat")
