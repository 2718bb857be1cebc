"""GPU tests of the sync-free, graph-replayed training step (step.FusedL1Step)
against the autograd path of the same loss (optim_to_render +
voxelize_gaussians_l1), which the other tests tie to the oracle and to the
reference. Tolerances: volume bit-exact (same kernels), loss 1e-5 relative,
gradients 1e-4 relative + 1e-4 of the array's max (atomic order)."""
import numpy as np
import pytest
import torch

from tests import _cases as K

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def grad_close(got, want, name):
    got, want = got.double().cpu().numpy(), want.double().cpu().numpy()
    tol = 1e-4 * np.abs(want) + 1e-4 * max(np.abs(want).max(), 1e-30)
    bad = np.abs(got - want) > tol
    assert not bad.any(), f"{name}: {bad.sum()} of {bad.size} out of tolerance"


def _autograd(cfg, target, plan=None, one_d=False):
    from gs_voxelizer_b200.losses import voxelize_gaussians_l1
    from gs_voxelizer_b200.optim_to_render import optim_to_render
    arrs = list(K.inputs(cfg))
    if one_d:
        arrs[3] = arrs[3].reshape(-1)
    leaves = [dev(a).requires_grad_(True) for a in arrs]
    pr, cq, tmin, tmax, _ = optim_to_render(*leaves, cfg.vol, cfg.world,
                                            cfg.center)
    denom = float(np.prod(cfg.vol) * cfg.channels)
    loss, vol = voxelize_gaussians_l1(pr, cq, leaves[3], cfg.vol, tmin, tmax,
                                      target, denom=denom, plan=plan)
    loss.backward()
    return float(loss), vol, [l.grad for l in leaves]


def _step(cfg, target, plan=None, one_d=False, use_graph=True):
    from gs_voxelizer_b200.step import FusedL1Step
    arrs = list(K.inputs(cfg))
    if one_d:
        arrs[3] = arrs[3].reshape(-1)
    params = [dev(a) for a in arrs]
    denom = float(np.prod(cfg.vol) * cfg.channels)
    return params, FusedL1Step(*params, cfg.vol, cfg.world, cfg.center, target,
                               denom=denom, plan=plan, use_graph=use_graph)


def _compare(step, params, want):
    loss_w, vol_w, grads_w = want
    assert torch.equal(step.volume, vol_w)
    for p, g, name in zip(params, grads_w, ("pos3d", "scale3d", "quat", "intensity")):
        assert p.grad is not None and p.grad.shape == g.shape, name
        grad_close(p.grad, g, name)


@pytest.mark.parametrize("channels,one_d,use_graph",
                         [(1, False, True), (1, True, True), (3, False, True),
                          (2, False, False)])
def test_step_matches_autograd(channels, one_d, use_graph):
    from gs_voxelizer_b200.workloads import phantom
    cfg = K.small_config(vol=(40, 36, 52), n=3000, seed=70, channels=channels,
                         scale=(0.005, 0.05))
    target = phantom(cfg, device="cuda")
    want = _autograd(cfg, target, one_d=one_d and channels == 1)
    params, step = _step(cfg, target, one_d=one_d and channels == 1,
                         use_graph=use_graph)
    for _ in range(3):  # replays give the same answer
        loss = step.run()
        assert loss == pytest.approx(want[0], rel=1e-5)
        _compare(step, params, want)
    assert step.regrows == 0


def test_step_follows_parameter_updates():
    """The graph reads the parameters in place: an in-place update changes
    the next step exactly as a fresh autograd evaluation does."""
    from gs_voxelizer_b200.workloads import phantom
    cfg = K.small_config(vol=(32, 32, 32), n=2000, seed=71, scale=(0.01, 0.04))
    target = phantom(cfg, device="cuda")
    params, step = _step(cfg, target)
    step.run()
    with torch.no_grad():
        for p in params:
            p.sub_(1e-3 * p.grad)
    loss = step.run()
    moved = [p.detach().cpu().numpy() for p in params]
    from gs_voxelizer_b200.losses import voxelize_gaussians_l1
    from gs_voxelizer_b200.optim_to_render import optim_to_render
    leaves = [dev(a).requires_grad_(True) for a in moved]
    pr, cq, tmin, tmax, _ = optim_to_render(*leaves, cfg.vol, cfg.world, cfg.center)
    want, vol = voxelize_gaussians_l1(pr, cq, leaves[3], cfg.vol, tmin, tmax, target)
    want.backward()
    assert loss == pytest.approx(float(want), rel=1e-5)
    assert torch.equal(step.volume, vol)
    for p, l, name in zip(params, leaves, ("pos3d", "scale3d", "quat", "intensity")):
        grad_close(p.grad, l.grad, name)


@pytest.mark.parametrize("use_graph", [True, False])
def test_step_overflow_grows_and_repeats(use_graph):
    """A pair buffer that is too small: the clamped step stays in bounds, the
    overflow is detected, the buffer grows and the step repeats with the
    correct result."""
    from gs_voxelizer_b200.workloads import phantom
    cfg = K.small_config(vol=(48, 40, 44), n=4000, seed=72, scale=(0.01, 0.06))
    target = phantom(cfg, device="cuda")
    want = _autograd(cfg, target)
    params, step = _step(cfg, target, use_graph=use_graph)
    true_count = int(step.count.item())
    assert true_count > 4 * 1024
    step._resize(0)  # capacity 1024, far below the count
    assert step.capacity < true_count
    loss = step.run()
    assert step.regrows == 1 and step.capacity >= true_count
    assert loss == pytest.approx(want[0], rel=1e-5)
    _compare(step, params, want)


def test_step_on_a_slab():
    """A z-slab plan without a process group: the slab's share of the loss
    and its gradients, as the autograd slab path computes them."""
    from gs_voxelizer_b200.slab import SlabPlan
    from gs_voxelizer_b200.workloads import phantom
    cfg = K.small_config(vol=(64, 40, 40), n=3000, seed=73, scale=(0.01, 0.05))
    plan = SlabPlan(cfg.vol, 2, 6)
    target = phantom(cfg, device="cuda", z_range=(plan.z_begin, plan.z_end))
    want = _autograd(cfg, target, plan=plan)
    params, step = _step(cfg, target, plan=plan)
    loss = step.run()
    assert loss == pytest.approx(want[0], rel=1e-5)
    _compare(step, params, want)


@pytest.mark.parametrize("force_overflow", [False, True])
def test_step_many_tiles(force_overflow):
    """More than 64K tiles (136 x 512 x 512 voxels = 69 632 tiles): the
    binning's multi-block scan path, including its pair count and overflow
    flag."""
    from gs_voxelizer_b200.workloads import phantom
    cfg = K.small_config(vol=(136, 512, 512), n=3000, seed=74,
                         scale=(0.002, 0.01))
    target = phantom(cfg, device="cuda")
    want = _autograd(cfg, target)
    params, step = _step(cfg, target)
    if force_overflow:
        step._resize(0)
    loss = step.run()
    assert step.regrows == (1 if force_overflow else 0)
    assert int(step.count.item()) <= step.capacity
    assert loss == pytest.approx(want[0], rel=1e-5)
    _compare(step, params, want)


@pytest.mark.parametrize("vol,channels,tz", [((19, 23, 29), 3, None),
                                             ((43, 17, 21), 1, (2, 6)),
                                             ((9, 8, 7), 4, None)])
def test_step_odd_shapes(vol, channels, tz):
    """Dimensions that are not multiples of 8 (or of 4): the fused loss's
    unaligned staging and epilogue paths; a slab ending in a partial tile
    layer."""
    from gs_voxelizer_b200.slab import SlabPlan
    from gs_voxelizer_b200.workloads import phantom
    cfg = K.small_config(vol=vol, n=1500, seed=75, channels=channels,
                         scale=(0.01, 0.08))
    plan = SlabPlan(cfg.vol, *tz) if tz else None
    zr = (plan.z_begin, plan.z_end) if plan else None
    target = phantom(cfg, device="cuda", z_range=zr)
    want = _autograd(cfg, target, plan=plan)
    params, step = _step(cfg, target, plan=plan)
    for _ in range(2):
        loss = step.run()
        assert loss == pytest.approx(want[0], rel=1e-5)
        _compare(step, params, want)
