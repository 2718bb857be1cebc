"""GPU parity: the CUDA path (through the C ABI, via gs_voxelizer_b200.cuda)
against the CPU oracle on the same seeded inputs.

Tolerances:
  * integers (tile_min/max, num_tiles_hit, gaussian_ids_sorted, tile_bins):
    bit-exact. For the projection, the oracle evaluates in IEEE float while
    the GPU uses the reference's fast-math arithmetic, so a tile bound whose
    pre-truncation value lies within 1e-5 (relative) of an integer may differ
    by one; those are counted and must be rare. Binning is compared on the
    GPU's own tile boxes and must match exactly.
  * volume: |gpu - oracle| <= 1e-5 * |oracle| + 1e-6.
  * gradients: |gpu - oracle| <= 1e-4 * |oracle| + 1e-4 * max|oracle| per
    output array (atomic summation order differs).
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests import _cases as K

pytestmark = pytest.mark.gpu

VOL_RTOL, VOL_ATOL = 1e-5, 1e-6
GRAD_RTOL, GRAD_ATOL_REL = 1e-4, 1e-4


def C():
    from gs_voxelizer_b200 import cuda as _C
    return _C


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t if dtype is None else t.to(dtype)


def host(t):
    return t.detach().cpu().numpy()


def assert_vol_close(got, ref):
    err = np.abs(got.astype(np.float64) - ref)
    bad = err > VOL_RTOL * np.abs(ref) + VOL_ATOL
    assert not bad.any(), (
        f"{bad.sum()} of {bad.size} voxels out of tolerance, max err "
        f"{err.max():.3e}")
    # where every contribution is culled the voxel is exactly zero (the
    # kernels cull by flushing to zero; a contribution exactly at the
    # threshold may fall either way, so allow a few)
    zero = ref == 0
    stray = int((got[zero] != 0).sum())
    assert stray <= max(2, zero.sum() // 10000), (stray, int(zero.sum()))


def assert_grad_close(got, ref, what):
    ref = ref.astype(np.float64)
    err = np.abs(got.astype(np.float64) - ref)
    tol = GRAD_RTOL * np.abs(ref) + GRAD_ATOL_REL * max(np.abs(ref).max(), 1e-30)
    bad = err > tol
    assert not bad.any(), (
        f"{what}: {bad.sum()} of {bad.size} out of tolerance, worst "
        f"err {err.max():.3e} (ref max {np.abs(ref).max():.3e})")


def project(cfg):
    pos, scale, quat, inten = K.inputs(cfg)
    out = C().optim_to_render_forward(cfg.n, dev(pos), dev(scale), dev(quat),
                                      dev(inten), cfg.vol, cfg.world, cfg.center)
    return (pos, scale, quat, inten), out


def bin_gpu(n, tmin, tmax, nt, vol):
    cum = torch.cumsum(nt, 0, dtype=torch.int32)
    n_isect = int(cum[-1].item()) if n else 0
    ids, bins = C().bin_and_sort_gaussians(n, n_isect, tmin, tmax, cum, vol)
    return ids, bins, n_isect


# ------------------------------------------------------------- projection

@pytest.mark.parametrize("channels", [1, 2, 3, 4])
def test_projection_parity(channels):
    cfg = K.small_config(vol=(60, 50, 70), n=3000, seed=21, channels=channels,
                         scale=(0.005, 0.05))
    (pos, scale, quat, inten), g = project(cfg)
    pr, cq, tmin, tmax, nt, bounds = O.optim_to_render_forward(
        pos, scale, quat, inten, cfg.vol, cfg.world, cfg.center,
        return_bounds=True)
    g = [host(t) for t in g]
    frac = np.abs(bounds - np.round(bounds))
    ambiguous = (frac < 1e-5 * np.maximum(1.0, np.abs(bounds))).any(axis=1)
    same = ((g[2] == tmin).all(1) & (g[3] == tmax).all(1) & (g[4] == nt))
    assert (same | ambiguous).all(), np.nonzero(~(same | ambiguous))[0][:10]
    assert (~same).sum() <= max(2, cfg.n // 1000)
    ok = same & (nt > 0)
    np.testing.assert_allclose(g[0][ok], pr[ok], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(g[1][ok], cq[ok], rtol=2e-3,
                               atol=2e-5 * np.abs(cq).max())
    culled = nt == 0
    assert not g[0][culled & same].any() and not g[1][culled & same].any()


def test_projection_backward_parity():
    cfg = K.small_config(vol=(40, 40, 40), n=2000, seed=22, scale=(0.01, 0.06))
    (pos, scale, quat, inten), g = project(cfg)
    pr_g = g[0]
    rng = np.random.default_rng(3)
    Gp = rng.standard_normal((cfg.n, 4)).astype(np.float32)
    Gc = rng.standard_normal((cfg.n, 6)).astype(np.float32)
    out = C().optim_to_render_backward(cfg.n, dev(pos), dev(scale), dev(quat),
                                       cfg.vol, cfg.world, cfg.center, dev(Gp),
                                       dev(Gc), pr_g)
    ref = O.optim_to_render_backward(pos, scale, quat, cfg.vol, cfg.world, Gp,
                                     Gc, host(pr_g))
    for got, want, name in zip(out, ref, ("pos", "scale", "quat")):
        assert_grad_close(host(got), want, name)


def test_pos3d_radii_buffer():
    """optim_to_render(..., pos3d_radii_buffer=buf) returns buf itself, filled
    with the projection, gradients flow through it, and a wrong buffer
    raises ValueError (gs_voxelizer/optim_to_render.py:98-113)."""
    from gs_voxelizer_b200.optim_to_render import optim_to_render
    cfg = K.small_config(vol=(24, 32, 40), n=500, seed=23)
    arrs = K.inputs(cfg)
    leaves = [dev(a).requires_grad_(True) for a in arrs]
    a = optim_to_render(*leaves, cfg.vol, cfg.world, cfg.center)
    buf = torch.empty((cfg.n, 4), device="cuda")
    leaves2 = [dev(x).requires_grad_(True) for x in arrs]
    b = optim_to_render(*leaves2, cfg.vol, cfg.world, cfg.center,
                        pos3d_radii_buffer=buf)
    assert b[0].data_ptr() == buf.data_ptr()
    assert torch.equal(a[0], b[0])
    (a[0].sum() + a[1].sum()).backward()
    (b[0].sum() + b[1].sum()).backward()
    for x, y in zip(leaves[:3], leaves2[:3]):
        assert torch.equal(x.grad, y.grad)
    for bad in (torch.empty((cfg.n, 3), device="cuda"),
                torch.empty((cfg.n, 4), device="cuda", dtype=torch.float64)):
        with pytest.raises(ValueError):
            optim_to_render(*leaves, cfg.vol, cfg.world, cfg.center,
                            pos3d_radii_buffer=bad)


# ---------------------------------------------------------------- binning

@pytest.mark.parametrize("vol,n,scale", [
    ((37, 29, 45), 800, (0.01, 0.08)),
    ((64, 64, 64), 5000, (0.002, 0.03)),
    ((9, 1, 17), 50, (0.01, 0.2)),
])
def test_binning_bit_exact(vol, n, scale):
    cfg = K.small_config(vol=vol, n=n, seed=23, scale=scale)
    _, (pr, cq, tmin, tmax, nt) = project(cfg)
    ids, bins, n_isect = bin_gpu(cfg.n, tmin, tmax, nt, cfg.vol)
    ids_o, bins_o = O.bin_and_sort_gaussians(host(tmin), host(tmax), cfg.vol)
    assert n_isect == ids_o.shape[0]
    np.testing.assert_array_equal(host(ids), ids_o)
    np.testing.assert_array_equal(host(bins), bins_o)


@pytest.mark.parametrize("n", [600, 20000])
def test_binning_large_segments(n):
    """Every Gaussian covers every tile: segments of n ids exercise the
    shared-memory (<= 16384) and the radix (> 16384) segment sorts."""
    vol = (16, 24, 16)
    cfg = K.small_config(vol=vol, n=n, seed=24, scale=(0.5, 0.6),
                         pos=(0.4, 0.6))
    _, (pr, cq, tmin, tmax, nt) = project(cfg)
    assert int(host(nt).min()) == 12
    ids, bins, n_isect = bin_gpu(cfg.n, tmin, tmax, nt, cfg.vol)
    ids_o, bins_o = O.bin_and_sort_gaussians(host(tmin), host(tmax), cfg.vol)
    np.testing.assert_array_equal(host(ids), ids_o)
    np.testing.assert_array_equal(host(bins), bins_o)


def test_binning_no_intersections():
    T = C().num_tiles((20, 20, 20))
    tmin = torch.zeros((10, 3), dtype=torch.int32, device="cuda")
    cum = torch.zeros((10,), dtype=torch.int32, device="cuda")
    ids, bins = C().bin_and_sort_gaussians(10, 0, tmin, tmin, cum, (20, 20, 20))
    assert ids.numel() == 0 and bins.shape == (T, 2)
    assert not host(bins).any()


# ------------------------------------------------------------ voxelization

def pipeline(cfg, per_gaussian=True, grad_seed=5):
    (pos, scale, quat, inten), (pr, cq, tmin, tmax, nt) = project(cfg)
    ids, bins, n_isect = bin_gpu(cfg.n, tmin, tmax, nt, cfg.vol)
    it = dev(inten)
    vol = C().voxelize_forward(cfg.vol, ids, bins, pr, cq, it)
    rng = np.random.default_rng(grad_seed)
    W = rng.standard_normal(tuple(vol.shape)).astype(np.float32)
    fn = (C().voxelize_backward_per_gaussian if per_gaussian
          else C().voxelize_backward)
    grads = fn(cfg.vol, ids, bins, pr, cq, it, dev(W))
    return dict(inten=inten, pr=host(pr), cq=host(cq), tmin=host(tmin),
                tmax=host(tmax), ids=host(ids), bins=host(bins),
                vol=host(vol), W=W, grads=[host(g) for g in grads])


@pytest.mark.parametrize("channels", [1, 2, 3, 4])
def test_forward_parity(channels):
    cfg = K.small_config(vol=(45, 38, 52), n=1500, seed=25, channels=channels,
                         scale=(0.005, 0.05))
    r = pipeline(cfg)
    ref = O.voxelize_forward(cfg.vol, r["ids"], r["bins"], r["pr"], r["cq"],
                             r["inten"])
    assert r["vol"].shape == ref.shape
    assert ref.max() > 0.1
    assert_vol_close(r["vol"], ref)


@pytest.mark.parametrize("channels", [1, 2, 3, 4])
@pytest.mark.parametrize("per_gaussian", [True, False])
def test_backward_parity(channels, per_gaussian):
    cfg = K.small_config(vol=(33, 40, 27), n=900, seed=26, channels=channels,
                         scale=(0.005, 0.06))
    r = pipeline(cfg, per_gaussian=per_gaussian)
    ref = O.voxelize_backward(cfg.vol, r["tmin"], r["tmax"], r["pr"], r["cq"],
                              r["inten"], r["W"])
    for got, want, name in zip(r["grads"], ref, ("pos", "conic", "intensity")):
        assert got.shape == want.shape
        assert_grad_close(got, want, name)
    assert not r["grads"][0][:, 3].any()


@pytest.mark.parametrize("channels", [1, 3])
@pytest.mark.parametrize("gscale", [1e25, 1e-25, 0.0])
def test_backward_gradient_magnitudes(channels, gscale):
    """dL/dvol far from unit scale moves the per-tile power-of-two staging
    scale to its limits (at 1e25 the kernel takes its exact path); half of
    the tiles get a zero gradient (their work items are skipped). Gradients
    are linear in dL/dvol, so the result is the oracle's, scaled."""
    cfg = K.small_config(vol=(33, 40, 27), n=900, seed=26, channels=channels,
                         scale=(0.005, 0.06))
    r = pipeline(cfg)
    W = r["W"].copy()
    W[: W.shape[0] // 2] = 0.0
    Ws = (W.astype(np.float64) * gscale).astype(np.float32)
    got = C().voxelize_backward_per_gaussian(
        cfg.vol, dev(r["ids"]), dev(r["bins"]), dev(r["pr"]), dev(r["cq"]),
        dev(r["inten"]), dev(Ws))
    ref = O.voxelize_backward(cfg.vol, r["tmin"], r["tmax"], r["pr"], r["cq"],
                              r["inten"], W)
    for g, want, name in zip(got, ref, ("pos", "conic", "intensity")):
        g = host(g)
        assert np.isfinite(g).all(), name
        if gscale == 0.0:
            assert not g.any(), name
        else:
            assert_grad_close(g.astype(np.float64) / gscale, want, name)


NEEDLE_RTOL = 2e-3


def needle_inputs():
    """Every third Gaussian squeezed 25:1 along x: det(Q) < 1e-5 tr(Q)^3, so
    it is not robustly positive definite and the kernels test the sign of
    sigma per voxel, as the reference does."""
    cfg = K.small_config(vol=(40, 40, 40), n=1200, seed=29, scale=(0.01, 0.05))
    pos, scale, quat, inten = K.inputs(cfg)
    scale = scale.copy()
    scale[::3, 0] *= 0.04
    return cfg, (pos, scale, quat, inten)


def test_needle_gaussians_exact_path():
    """Needles mixed with ordinary Gaussians in the same tiles and work
    items. Such Gaussians are ill-conditioned: sigma is a sum of terms ~600x
    larger than itself, so every float32 evaluation order differs. Measured
    here on this input, the reference's own CUDA forward differs from the
    IEEE-float oracle by up to 4.5e-4 relative; hence NEEDLE_RTOL for the
    volume and 10x the usual relative tolerance for the gradients."""
    cfg, (pos, scale, quat, inten) = needle_inputs()
    pr, cq, tmin, tmax, nt = C().optim_to_render_forward(
        cfg.n, dev(pos), dev(scale), dev(quat), dev(inten), cfg.vol, cfg.world,
        cfg.center)
    q = host(cq).astype(np.float64)
    a, b, c, d, e, f = q.T
    det = a * (d * f - e * e) - b * (b * f - e * c) + c * (b * e - d * c)
    tr = a + d + f
    live = host(nt) > 0
    assert (live & ~(det >= 1e-5 * tr ** 3)).sum() > 20  # non-robust, drawn
    ids, bins, _ = bin_gpu(cfg.n, tmin, tmax, nt, cfg.vol)
    it = dev(inten)
    vol = C().voxelize_forward(cfg.vol, ids, bins, pr, cq, it)
    ref = O.voxelize_forward(cfg.vol, host(ids), host(bins), host(pr),
                             host(cq), inten)
    err = np.abs(host(vol).astype(np.float64) - ref)
    assert (err <= NEEDLE_RTOL * np.abs(ref) + VOL_ATOL).all(), err.max()
    W = np.random.default_rng(4).standard_normal(tuple(vol.shape)).astype(np.float32)
    got = C().voxelize_backward_per_gaussian(cfg.vol, ids, bins, pr, cq, it,
                                             dev(W))
    gref = O.voxelize_backward(cfg.vol, host(tmin), host(tmax), host(pr),
                               host(cq), inten, W)
    for g, want, name in zip(got, gref, ("pos", "conic", "intensity")):
        want = want.astype(np.float64)
        e = np.abs(host(g).astype(np.float64) - want)
        tol = 10 * GRAD_RTOL * np.abs(want) + GRAD_ATOL_REL * np.abs(want).max()
        assert (e <= tol).all(), (name, (e > tol).sum())


@pytest.mark.parametrize("vol", [(1, 1, 1), (8, 8, 8), (17, 3, 9), (5, 70, 12)])
def test_odd_volumes(vol):
    cfg = K.small_config(vol=vol, n=40, seed=27, scale=(0.05, 0.3))
    r = pipeline(cfg)
    ref = O.voxelize_forward(cfg.vol, r["ids"], r["bins"], r["pr"], r["cq"],
                             r["inten"])
    assert_vol_close(r["vol"], ref)
    gref = O.voxelize_backward(cfg.vol, r["tmin"], r["tmax"], r["pr"], r["cq"],
                               r["inten"], r["W"])
    for got, want, name in zip(r["grads"], gref, ("pos", "conic", "intensity")):
        assert_grad_close(got, want, name)


def test_forward_deterministic():
    cfg = K.small_config(vol=(64, 64, 64), n=4000, seed=28, scale=(0.005, 0.04))
    (pos, scale, quat, inten), (pr, cq, tmin, tmax, nt) = project(cfg)
    ids, bins, _ = bin_gpu(cfg.n, tmin, tmax, nt, cfg.vol)
    a = C().voxelize_forward(cfg.vol, ids, bins, pr, cq, dev(inten))
    b = C().voxelize_forward(cfg.vol, ids, bins, pr, cq, dev(inten))
    assert torch.equal(a, b)


def test_all_culled_gives_zeros():
    cfg = K.small_config(vol=(20, 20, 20), n=30, seed=29)
    pos, scale, quat, inten = K.inputs(cfg)
    pos = pos + 10.0  # everything outside the volume
    from gs_voxelizer_b200.optim_to_render import optim_to_render
    from gs_voxelizer_b200.voxelize import voxelize_gaussians
    p = dev(pos).requires_grad_(True)
    out = optim_to_render(p, dev(scale), dev(quat), dev(inten), cfg.vol,
                          cfg.world, cfg.center)
    vol = voxelize_gaussians(out[0], out[1], dev(inten), cfg.vol, out[2],
                             out[3], out[4])
    assert vol.shape == (20, 20, 20, 1) and not vol.any()
    vol.sum().backward()
    assert not p.grad.any()


# ------------------------------------------------------------ end to end

@pytest.mark.parametrize("per_gaussian", [True, False])
def test_autograd_chain_matches_oracle(per_gaussian):
    """optim_to_render -> voxelize_gaussians -> L1 loss -> backward through
    the public API, against the oracle's explicit chain."""
    from gs_voxelizer_b200.optim_to_render import optim_to_render
    from gs_voxelizer_b200.voxelize import voxelize_gaussians
    from gs_voxelizer_b200.workloads import phantom

    cfg = K.small_config(vol=(48, 40, 56), n=2500, seed=30, channels=2,
                         scale=(0.005, 0.04))
    pos, scale, quat, inten = K.inputs(cfg)
    target = phantom(cfg, device="cuda")
    leaves = [dev(a).requires_grad_(True) for a in (pos, scale, quat, inten)]
    pr, cq, tmin, tmax, nt = optim_to_render(*leaves, cfg.vol, cfg.world,
                                             cfg.center)
    vol = voxelize_gaussians(pr, cq, leaves[3], cfg.vol, tmin, tmax, nt,
                             use_per_gaussian_backward=per_gaussian)
    loss = torch.nn.functional.l1_loss(vol, target)
    loss.backward()

    pr_h, cq_h = host(pr), host(cq)
    ids, bins = O.bin_and_sort_gaussians(host(tmin), host(tmax), cfg.vol)
    vol_o = O.voxelize_forward(cfg.vol, ids, bins, pr_h, cq_h, inten)
    assert_vol_close(host(vol), vol_o)
    loss_o, g = O.l1_loss_and_grad(vol_o, host(target))
    assert float(loss) == pytest.approx(loss_o, rel=1e-5)
    # the oracle chain uses the GPU's dL/dvol so that sign flips at
    # |vol - target| ~ 0 do not enter the comparison
    g = np.sign(host(vol) - host(target)) / vol_o.size
    gp, gc, gi = O.voxelize_backward(cfg.vol, host(tmin), host(tmax), pr_h,
                                     cq_h, inten, g.astype(np.float32))
    dpos, dscale, dquat = O.optim_to_render_backward(pos, scale, quat, cfg.vol,
                                                     cfg.world, gp, gc, pr_h)
    assert_grad_close(host(leaves[0].grad), dpos, "pos3d")
    assert_grad_close(host(leaves[1].grad), dscale, "scale3d")
    assert_grad_close(host(leaves[2].grad), dquat, "quat")
    assert_grad_close(host(leaves[3].grad), gi, "intensity")


# ------------------------------------------------------------------ slabs

def test_slab_path_matches_full():
    from gs_voxelizer_b200 import slab

    cfg = K.small_config(vol=(70, 33, 41), n=2000, seed=31, scale=(0.005, 0.05))
    (pos, scale, quat, inten), (pr, cq, tmin, tmax, nt) = project(cfg)
    ids, bins, _ = bin_gpu(cfg.n, tmin, tmax, nt, cfg.vol)
    it = dev(inten)
    full = C().voxelize_forward(cfg.vol, ids, bins, pr, cq, it)
    W = torch.randn(full.shape, device="cuda", generator=torch.Generator("cuda").manual_seed(1))
    gfull = C().voxelize_backward_per_gaussian(cfg.vol, ids, bins, pr, cq, it, W)
    Tz = (cfg.vol[0] + 7) // 8
    acc = [torch.zeros_like(g) for g in gfull]
    tpl = ((cfg.vol[1] + 7) // 8) * ((cfg.vol[2] + 7) // 8)
    bins_h = host(bins)
    for tz0, tz1 in ((0, 3), (3, 4), (4, Tz)):
        s = slab.SlabPlan(cfg.vol, tz0, tz1)
        sids, sbins = s.bin(tmin, tmax)
        full_b = bins_h[tz0 * tpl:tz1 * tpl]
        nz = full_b[:, 1] > full_b[:, 0]
        if nz.any():
            start = full_b[nz][0, 0]
            np.testing.assert_array_equal(host(sbins)[nz], full_b[nz] - start)
            np.testing.assert_array_equal(host(sids), host(ids)[start:full_b[nz][-1, 1]])
        svol = s.forward(sids, sbins, pr, cq, it)
        assert torch.equal(svol, full[s.z_begin:s.z_end])
        sg = s.backward(sids, sbins, pr, cq, it, W[s.z_begin:s.z_end].contiguous())
        for a, b in zip(acc, sg):
            a += b
    for got, want, name in zip(acc, gfull, ("pos", "conic", "intensity")):
        assert_grad_close(host(got), host(want), name)


# ------------------------------------------------------- full-size checks

def test_full_size_step256_properties():
    """BASELINE configuration 2 at full size (256^3, 100k Gaussians):
    size-independent properties everywhere plus an oracle check on a slab."""
    from gs_voxelizer_b200 import slab
    from gs_voxelizer_b200.workloads import CONFIGS

    cfg = CONFIGS["step256"]
    (pos, scale, quat, inten), (pr, cq, tmin, tmax, nt) = project(cfg)
    ids, bins, n_isect = bin_gpu(cfg.n, tmin, tmax, nt, cfg.vol)
    b = host(bins).astype(np.int64)
    cnt = b[:, 1] - b[:, 0]
    assert cnt.sum() == n_isect == int(host(nt).sum())
    idh = host(ids)
    nz = np.nonzero(cnt)[0]
    # ranges are contiguous and ascending, ids strictly increase inside tiles
    assert (b[nz[1:], 0] == b[nz[:-1], 1]).all()
    d = np.diff(idh)
    boundaries = np.zeros(n_isect, bool)
    boundaries[b[nz, 0]] = True
    assert (d[~boundaries[1:]] > 0).all()
    it = dev(inten)
    vol = C().voxelize_forward(cfg.vol, ids, bins, pr, cq, it)
    assert torch.isfinite(vol).all() and float(vol.min()) >= 0.0
    # oracle on two tile layers in the middle of the volume
    s = slab.SlabPlan(cfg.vol, 15, 17)
    sids, sbins = s.bin(tmin, tmax)
    ref = O.voxelize_forward(cfg.vol, host(sids), host(sbins), host(pr),
                             host(cq), inten, tile_z=(15, 17))
    assert_vol_close(host(vol[s.z_begin:s.z_end]), ref)
