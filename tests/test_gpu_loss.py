"""GPU tests of the L1 loss kernels, standalone and fused into voxelization.
Tolerances: loss 1e-5 relative (float reduction order), gradients as in
test_gpu_parity (1e-4 relative + 1e-4 of the array's max)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests import _cases as K

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    return t.detach().cpu().numpy()


def grad_close(got, want, name):
    got, want = host(got).astype(np.float64), host(want).astype(np.float64)
    tol = 1e-4 * np.abs(want) + 1e-4 * max(np.abs(want).max(), 1e-30)
    bad = np.abs(got - want) > tol
    assert not bad.any(), f"{name}: {bad.sum()} of {bad.size} out of tolerance"


@pytest.mark.parametrize("shape", [(37, 41, 29, 1), (16, 16, 16, 4), (7,)])
def test_l1_loss_matches_torch(shape):
    from gs_voxelizer_b200.losses import l1_loss
    g = torch.Generator("cuda").manual_seed(0)
    v = torch.randn(shape, device="cuda", generator=g).requires_grad_(True)
    t = torch.randn(shape, device="cuda", generator=g)
    v2 = v.detach().clone().requires_grad_(True)
    a = l1_loss(v, t)
    b = torch.nn.functional.l1_loss(v2, t)
    assert float(a) == pytest.approx(float(b), rel=1e-5)
    (3.0 * a).backward()
    (3.0 * b).backward()
    torch.testing.assert_close(v.grad, v2.grad, rtol=1e-6, atol=0)
    s = l1_loss(v.detach(), t, reduction="sum")
    assert float(s) == pytest.approx(float((v.detach() - t).abs().sum()), rel=1e-5)


def _setup(cfg):
    from gs_voxelizer_b200.optim_to_render import optim_to_render
    from gs_voxelizer_b200.workloads import phantom
    pos, scale, quat, inten = K.inputs(cfg)
    target = phantom(cfg, device="cuda")
    leaves = [dev(a).requires_grad_(True) for a in (pos, scale, quat, inten)]
    proj = optim_to_render(*leaves, cfg.vol, cfg.world, cfg.center)
    return leaves, proj, target


@pytest.mark.parametrize("channels", [1, 3])
def test_fused_voxelize_l1_matches_unfused(channels):
    from gs_voxelizer_b200.losses import voxelize_gaussians_l1
    from gs_voxelizer_b200.voxelize import voxelize_gaussians
    cfg = K.small_config(vol=(40, 36, 52), n=2000, seed=50, channels=channels,
                         scale=(0.005, 0.05))
    leaves, (pr, cq, tmin, tmax, nt), target = _setup(cfg)
    loss, vol = voxelize_gaussians_l1(pr, cq, leaves[3], cfg.vol, tmin, tmax,
                                      target)
    loss.backward()
    fused = [l.grad.clone() for l in leaves]
    for l in leaves:
        l.grad = None

    leaves2, (pr2, cq2, tmin2, tmax2, nt2), _ = _setup(cfg)
    vol2 = voxelize_gaussians(pr2, cq2, leaves2[3], cfg.vol, tmin2, tmax2, nt2)
    loss2 = torch.nn.functional.l1_loss(vol2, target)
    loss2.backward()
    assert torch.equal(vol, vol2.detach())
    assert float(loss) == pytest.approx(float(loss2), rel=1e-5)
    for a, b, name in zip(fused, [l.grad for l in leaves2],
                          ("pos3d", "scale3d", "quat", "intensity")):
        grad_close(a, b, name)
    # and against the oracle's loss
    ids, bins = O.bin_and_sort_gaussians(host(tmin), host(tmax), cfg.vol)
    vo = O.voxelize_forward(cfg.vol, ids, bins, host(pr), host(cq), K.inputs(cfg)[3])
    lo, _ = O.l1_loss_and_grad(vo, host(target))
    assert float(loss) == pytest.approx(lo, rel=1e-5)


def test_fused_l1_slabs_sum_to_full():
    from gs_voxelizer_b200.losses import voxelize_gaussians_l1
    from gs_voxelizer_b200.slab import SlabPlan
    cfg = K.small_config(vol=(60, 30, 34), n=1500, seed=51, scale=(0.005, 0.05))
    leaves, (pr, cq, tmin, tmax, nt), target = _setup(cfg)
    full, _ = voxelize_gaussians_l1(pr, cq, leaves[3], cfg.vol, tmin, tmax, target)
    full.backward(retain_graph=True)
    gfull = [l.grad.clone() for l in leaves]
    for l in leaves:
        l.grad = None
    total = 0.0
    for tz0, tz1 in ((0, 3), (3, 5), (5, 8)):
        plan = SlabPlan(cfg.vol, tz0, tz1)
        part, _ = voxelize_gaussians_l1(pr, cq, leaves[3], cfg.vol, tmin, tmax,
                                        target[plan.z_begin:plan.z_end], plan=plan)
        part.backward(retain_graph=True)
        total += float(part)
    assert total == pytest.approx(float(full), rel=1e-5)
    for a, b, name in zip([l.grad for l in leaves], gfull,
                          ("pos3d", "scale3d", "quat", "intensity")):
        grad_close(a, b, name)


def test_fused_l1_without_intersections():
    from gs_voxelizer_b200.losses import voxelize_gaussians_l1
    cfg = K.small_config(vol=(20, 20, 20), n=10, seed=52)
    leaves, _, target = _setup(cfg)
    pr = torch.zeros((10, 4), device="cuda")
    cq = torch.zeros((10, 6), device="cuda")
    tm = torch.zeros((10, 3), dtype=torch.int32, device="cuda")
    loss, vol = voxelize_gaussians_l1(pr, cq, leaves[3], cfg.vol, tm, tm, target)
    assert not vol.any()
    assert float(loss) == pytest.approx(float(target.abs().mean()), rel=1e-6)
