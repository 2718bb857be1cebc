"""CPU checks of the oracle (oracle/gsv_oracle.c) against independent float64
restatements, finite differences and the reference's published semantics.
No GPU needed."""
import numpy as np
import pytest

from oracle import oracle as O
from tests import _cases as K


def _project(cfg):
    pos, scale, quat, inten = K.inputs(cfg)
    out = O.optim_to_render_forward(pos, scale, quat, inten, cfg.vol, cfg.world,
                                    cfg.center, return_bounds=True)
    return (pos, scale, quat, inten), out


@pytest.mark.parametrize("channels", [1, 3])
def test_projection_matches_float64(channels):
    cfg = K.small_config(n=400, channels=channels, seed=3)
    (pos, scale, quat, inten), (pr, cq, tmin, tmax, nt, bounds) = _project(cfg)
    live = nt > 0
    assert live.sum() > 300
    cov = K.voxel_cov64(scale, quat, cfg.vol, cfg.world)
    q64 = K.conic_from_cov(cov)
    np.testing.assert_allclose(cq[live], q64[live], rtol=2e-3, atol=1e-5)
    p64 = K.pixel_pos64(pos, cfg.vol, cfg.world, cfg.center)
    np.testing.assert_allclose(pr[live, :3], p64[live], rtol=1e-5, atol=1e-4)
    # tile boxes: integers from the float bounds (unambiguous ones only)
    mean = inten.astype(np.float64).mean(axis=1)
    ext = np.minimum(3.0, np.sqrt(2.0 * np.log(mean * 1e6)))
    r3 = np.maximum(0.0, np.sqrt(np.diagonal(cov, axis1=1, axis2=2)) * ext[:, None] - 0.5)
    lo64, hi64 = (p64 - r3) / 8.0, (p64 + r3 + 7.0) / 8.0
    Z, Y, X = cfg.vol
    bound = np.array([(X + 7) // 8, (Y + 7) // 8, (Z + 7) // 8])
    lo_i = np.clip(np.trunc(lo64), 0, bound).astype(np.int32)
    hi_i = np.clip(np.trunc(hi64), 0, bound).astype(np.int32)
    near = (np.abs(lo64 - np.round(lo64)) < 1e-4).any(1) | (np.abs(hi64 - np.round(hi64)) < 1e-4).any(1)
    sel = live & ~near
    np.testing.assert_array_equal(tmin[sel], lo_i[sel])
    np.testing.assert_array_equal(tmax[sel], hi_i[sel])
    np.testing.assert_array_equal(nt, np.prod(tmax - tmin, axis=1) * live)


def test_projection_culls():
    cfg = K.small_config(n=8, seed=1)
    pos, scale, quat, inten = K.inputs(cfg)
    pos = pos.copy(); scale = scale.copy(); inten = inten.copy(); quat = quat.copy()
    pos[0] = (5.0, 5.0, 5.0)           # far outside the volume
    scale[1] = (0.0, 0.02, 0.02)       # singular covariance: det == 0
    quat[1] = (1.0, 0.0, 0.0, 0.0)
    scale[2] = (0.0, 0.0, 0.0)         # radius 0
    inten[3] = 0.0                     # extent from log(0): still binned
    pr, cq, tmin, tmax, nt = O.optim_to_render_forward(
        pos, scale, quat, inten, cfg.vol, cfg.world, cfg.center)
    for g in (0, 1, 2):
        assert nt[g] == 0 and not pr[g].any() and not cq[g].any()
        assert not tmin[g].any() and not tmax[g].any()
    assert nt[4:].min() > 0


def test_binning_matches_stable_sort():
    cfg = K.small_config(vol=(37, 29, 45), n=250, seed=5, scale=(0.01, 0.08))
    _, (pr, cq, tmin, tmax, nt, _) = _project(cfg)
    ids, bins = O.bin_and_sort_gaussians(tmin, tmax, cfg.vol)
    ids_ref, bins_ref = K.stable_binning(tmin, tmax, cfg.vol)
    assert ids.shape[0] == int(nt.sum())
    np.testing.assert_array_equal(ids, ids_ref)
    np.testing.assert_array_equal(bins, bins_ref)


def test_binning_slabs_partition_the_full_binning():
    cfg = K.small_config(vol=(64, 40, 40), n=300, seed=6, scale=(0.01, 0.06))
    _, (pr, cq, tmin, tmax, nt, _) = _project(cfg)
    ids, bins = O.bin_and_sort_gaussians(tmin, tmax, cfg.vol)
    tpl = ((40 + 7) // 8) ** 2
    for tz0, tz1 in ((0, 3), (3, 5), (5, 8)):
        sids, sbins = O.bin_and_sort_gaussians(tmin, tmax, cfg.vol, tile_z=(tz0, tz1))
        full = bins[tz0 * tpl:tz1 * tpl]
        nz = full[:, 1] > full[:, 0]
        start = full[nz][0, 0]
        np.testing.assert_array_equal(sbins[nz], full[nz] - start)
        np.testing.assert_array_equal(sids, ids[start:full[nz][-1, 1]])


@pytest.mark.parametrize("channels", [1, 2, 4])
def test_forward_matches_float64(channels):
    cfg = K.small_config(vol=(24, 20, 28), n=120, seed=7, channels=channels,
                         scale=(0.02, 0.08))
    _, (pr, cq, tmin, tmax, nt, _) = _project(cfg)
    _, _, _, inten = K.inputs(cfg)
    ids, bins = O.bin_and_sort_gaussians(tmin, tmax, cfg.vol)
    vol = O.voxelize_forward(cfg.vol, ids, bins, pr, cq, inten)
    ref = K.forward64(cfg.vol, ids, bins, pr, cq, inten)
    assert vol.shape == (*cfg.vol, channels)
    assert vol.max() > 0.1
    np.testing.assert_allclose(vol, ref, rtol=1e-5, atol=2e-6)


def test_forward_slab_equals_full_slice():
    cfg = K.small_config(vol=(30, 24, 24), n=100, seed=8, scale=(0.02, 0.08))
    (_, _, _, inten), (pr, cq, tmin, tmax, nt, _) = _project(cfg)
    ids, bins = O.bin_and_sort_gaussians(tmin, tmax, cfg.vol)
    full = O.voxelize_forward(cfg.vol, ids, bins, pr, cq, inten)
    for tz0, tz1 in ((0, 2), (2, 4)):
        sids, sbins = O.bin_and_sort_gaussians(tmin, tmax, cfg.vol, tile_z=(tz0, tz1))
        part = O.voxelize_forward(cfg.vol, sids, sbins, pr, cq, inten, tile_z=(tz0, tz1))
        np.testing.assert_array_equal(part, full[8 * tz0:min(30, 8 * tz1)])


def _loss64(vol, ids, bins, pr, cq, inten, W):
    return float((K.forward64(vol, ids, bins, pr, cq, inten) * W).sum())


@pytest.mark.parametrize("channels", [1, 2])
def test_voxelize_backward_finite_differences(channels):
    cfg = K.small_config(vol=(16, 16, 24), n=6, seed=9, channels=channels,
                         scale=(0.06, 0.1), intensity=(0.5, 1.0))
    (_, _, _, inten), (pr, cq, tmin, tmax, nt, _) = _project(cfg)
    ids, bins = O.bin_and_sort_gaussians(tmin, tmax, cfg.vol)
    rng = np.random.default_rng(0)
    W = rng.standard_normal((*cfg.vol, channels)).astype(np.float32)
    gp, gc, gi = O.voxelize_backward(cfg.vol, tmin, tmax, pr, cq, inten, W)
    pr64, cq64, in64 = pr.astype(np.float64), cq.astype(np.float64), inten.astype(np.float64)
    eps = 1e-6
    for g in range(cfg.n):
        if nt[g] == 0:
            continue
        for k in range(3):
            a, b = pr64.copy(), pr64.copy()
            a[g, k] += eps; b[g, k] -= eps
            fd = (_loss64(cfg.vol, ids, bins, a, cq64, in64, W)
                  - _loss64(cfg.vol, ids, bins, b, cq64, in64, W)) / (2 * eps)
            assert gp[g, k] == pytest.approx(fd, rel=2e-3, abs=2e-3)
        for k in range(6):
            a, b = cq64.copy(), cq64.copy()
            a[g, k] += eps; b[g, k] -= eps
            fd = (_loss64(cfg.vol, ids, bins, pr64, a, in64, W)
                  - _loss64(cfg.vol, ids, bins, pr64, b, in64, W)) / (2 * eps)
            # off-diagonal conic entries appear twice in d^T Q d; the
            # reference's gradient is with respect to the stored entry
            assert gc[g, k] == pytest.approx(fd, rel=2e-3, abs=2e-3)
        for c in range(channels):
            a, b = in64.copy(), in64.copy()
            a[g, c] += eps; b[g, c] -= eps
            fd = (_loss64(cfg.vol, ids, bins, pr64, cq64, a, W)
                  - _loss64(cfg.vol, ids, bins, pr64, cq64, b, W)) / (2 * eps)
            assert gi[g, c] == pytest.approx(fd, rel=2e-3, abs=2e-3)
        assert gp[g, 3] == 0.0


def _conic_loss(scale, quat, vol, world, G):
    return float((K.conic_from_cov(K.voxel_cov64(scale, quat, vol, world)) * G).sum())


def test_projection_backward_finite_differences_and_quirk():
    cfg = K.small_config(vol=(32, 32, 32), n=5, seed=11, scale=(0.03, 0.08))
    pos, scale, quat, inten = K.inputs(cfg)
    pr, cq, tmin, tmax, nt = O.optim_to_render_forward(
        pos, scale, quat, inten, cfg.vol, cfg.world, cfg.center)
    rng = np.random.default_rng(1)
    G = rng.standard_normal((cfg.n, 6)).astype(np.float32)
    Gp = rng.standard_normal((cfg.n, 4)).astype(np.float32)
    gp, gs, gq = O.optim_to_render_backward(pos, scale, quat, cfg.vol, cfg.world,
                                            Gp, G, pr)
    # position: the reference multiplies by the voxel size (its quirk)
    vox = np.array([1 / 32, 1 / 32, 1 / 32], np.float32)
    np.testing.assert_allclose(gp, Gp[:, :3] * vox, rtol=1e-6)
    s64, q64, G64 = scale.astype(np.float64), quat.astype(np.float64), G.astype(np.float64)
    eps = 1e-7
    for g in range(cfg.n):
        Gg = np.zeros_like(G64); Gg[g] = G64[g]
        for k in range(3):
            a, b = s64.copy(), s64.copy()
            a[g, k] += eps; b[g, k] -= eps
            fd = (_conic_loss(a, q64, cfg.vol, cfg.world, Gg)
                  - _conic_loss(b, q64, cfg.vol, cfg.world, Gg)) / (2 * eps)
            assert gs[g, k] == pytest.approx(fd, rel=5e-3, abs=1e-3 * abs(fd) + 1e-3)
        # quaternion: gradient w.r.t. the normalised quaternion; compare the
        # component tangent to the unit sphere
        fdq = np.zeros(4)
        for k in range(4):
            a, b = q64.copy(), q64.copy()
            a[g, k] += eps; b[g, k] -= eps
            fdq[k] = (_conic_loss(s64, a, cfg.vol, cfg.world, Gg)
                      - _conic_loss(s64, b, cfg.vol, cfg.world, Gg)) / (2 * eps)
        u = q64[g] / np.linalg.norm(q64[g])
        proj = gq[g] - u * (u @ gq[g])
        np.testing.assert_allclose(proj, fdq, rtol=5e-3, atol=1e-3 * np.abs(fdq).max() + 1e-3)


def test_l1_loss_and_grad():
    rng = np.random.default_rng(2)
    v = rng.standard_normal((5, 6, 7, 1)).astype(np.float32)
    t = rng.standard_normal((5, 6, 7, 1)).astype(np.float32)
    loss, g = O.l1_loss_and_grad(v, t)
    assert loss == pytest.approx(np.abs(v - t).mean(), rel=1e-6)
    np.testing.assert_allclose(g, np.sign(v - t) / v.size, rtol=1e-6)
