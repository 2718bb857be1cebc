"""GPU tests of the 3D SSIM and TV losses (csrc/ssim.cu, losses.fused_ssim3d
and losses.tv3d), through the C ABI.

Checkers: the C oracle (float64, pinned on the CPU by
tests/test_ssim_tv_cpu.py) and a plain PyTorch float32 restatement (conv3d
with the separable window; autograd for the gradient). Tolerances: value
1e-5 relative (float32 sums over up to 2^21 voxels); gradients 1e-4
relative + 1e-4 of the array's max (float32 window sums in a different
order). The last test runs the reference's own training-step shape:
voxelize_gaussians -> fused_ssim3d on [1, 1, Z, Y, X] -> backward to the
Gaussian parameters, against the same chain with the torch SSIM."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests import _cases as K

pytestmark = pytest.mark.gpu


def close(got, want, name, rtol=1e-4, atol_rel=1e-4):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    tol = rtol * np.abs(want) + atol_rel * max(np.abs(want).max(), 1e-30)
    bad = np.abs(got - want) > tol
    assert not bad.any(), (f"{name}: {bad.sum()} of {bad.size} out of tolerance, "
                           f"max err {np.abs(got - want).max():.3e}")


@pytest.fixture(autouse=True)
def _no_tf32():
    """conv3d of the torch restatement in true float32 (cuDNN would use
    TF32 by default)."""
    prev = torch.backends.cudnn.allow_tf32
    torch.backends.cudnn.allow_tf32 = False
    yield
    torch.backends.cudnn.allow_tf32 = prev


def torch_ssim3d(a, b, c1=0.01 ** 2, c2=0.03 ** 2):
    """Plain PyTorch float32 3D SSIM: separable Gaussian window by conv3d,
    zero padding, mean over voxels and channels."""
    w = torch.tensor(O.ssim_window(), dtype=torch.float32, device=a.device)
    shape = a.shape
    x = a.reshape(-1, 1, *shape[-3:])
    y = b.reshape(-1, 1, *shape[-3:])

    def blur(v):
        v = torch.nn.functional.conv3d(v, w.view(1, 1, 1, 1, 11), padding=(0, 0, 5))
        v = torch.nn.functional.conv3d(v, w.view(1, 1, 1, 11, 1), padding=(0, 5, 0))
        return torch.nn.functional.conv3d(v, w.view(1, 1, 11, 1, 1), padding=(5, 0, 0))

    mx, my = blur(x), blur(y)
    sxx = blur(x * x) - mx * mx
    syy = blur(y * y) - my * my
    sxy = blur(x * y) - mx * my
    s = ((2 * mx * my + c1) * (2 * sxy + c2)) / ((mx * mx + my * my + c1) * (sxx + syy + c2))
    return s.mean()


def torch_tv3d(x, iso=True, eps=1e-8):
    dx = torch.zeros_like(x)
    dy = torch.zeros_like(x)
    dz = torch.zeros_like(x)
    dx[..., :, :, :-1] = x[..., :, :, 1:] - x[..., :, :, :-1]
    dy[..., :, :-1, :] = x[..., :, 1:, :] - x[..., :, :-1, :]
    dz[..., :-1, :, :] = x[..., 1:, :, :] - x[..., :-1, :, :]
    if iso:
        return torch.sqrt(dx * dx + dy * dy + dz * dz + eps).mean()
    return (dx.abs() + dy.abs() + dz.abs()).mean()


def _pair(shape, seed):
    g = torch.Generator("cuda").manual_seed(seed)
    a = torch.rand(shape, device="cuda", generator=g)
    b = (a + 0.2 * torch.randn(shape, device="cuda", generator=g)).clamp(0, 1)
    return a, b


SHAPES = [(1, 1, 37, 41, 29), (2, 3, 16, 16, 16), (40, 50, 33), (5, 3, 70)]


@pytest.mark.parametrize("shape", SHAPES)
def test_ssim3d_against_oracle(shape):
    from gs_voxelizer_b200.losses import fused_ssim3d
    a, b = _pair(shape, sum(shape))
    a.requires_grad_(True)
    v = fused_ssim3d(a, b)
    v.backward()
    want, gw = O.ssim3d(a.detach().cpu().numpy(), b.cpu().numpy())
    assert float(v.detach()) == pytest.approx(want, rel=1e-5)
    close(a.grad.cpu().numpy(), gw, "d ssim / d img1")


def test_ssim3d_against_torch_at_128():
    from gs_voxelizer_b200.losses import fused_ssim3d
    a, b = _pair((1, 1, 128, 128, 128), 7)
    a1 = a.clone().requires_grad_(True)
    a2 = a.clone().requires_grad_(True)
    v1 = fused_ssim3d(a1, b)
    (3.0 * v1).backward()
    v2 = torch_ssim3d(a2, b)
    (3.0 * v2).backward()
    assert float(v1) == pytest.approx(float(v2), rel=1e-5)
    close(a1.grad.cpu().numpy(), a2.grad.cpu().numpy(), "grad vs torch")


def test_ssim3d_identical_is_one():
    from gs_voxelizer_b200.losses import fused_ssim3d
    a, _ = _pair((33, 20, 47), 8)
    assert float(fused_ssim3d(a, a)) == pytest.approx(1.0, abs=1e-6)


@pytest.mark.parametrize("iso", [True, False])
@pytest.mark.parametrize("shape", [(2, 37, 41, 29), (64, 64, 64), (1, 1, 9)])
def test_tv3d_against_oracle_and_torch(iso, shape):
    from gs_voxelizer_b200.losses import tv3d
    x, _ = _pair(shape, 11 + len(shape))
    x1 = x.clone().requires_grad_(True)
    v = tv3d(x1, isotropic=iso)
    (2.0 * v).backward()
    want, gw = O.tv3d(x.cpu().numpy(), isotropic=iso)
    assert float(v) == pytest.approx(want, rel=1e-5)
    close(x1.grad.cpu().numpy(), 2.0 * gw, "d tv / dx")
    x2 = x.clone().requires_grad_(True)
    t = torch_tv3d(x2, iso)
    (2.0 * t).backward()
    assert float(v) == pytest.approx(float(t), rel=1e-5)
    if iso:  # |.| has a kink at 0 where torch's subgradient may differ
        close(x1.grad.cpu().numpy(), x2.grad.cpu().numpy(), "tv grad vs torch")


def test_voxelize_then_ssim_step_gradients():
    """The reference's test flow (test/test_gs_voxelizer.py:50-70):
    optim_to_render -> voxelize_gaussians -> fused_ssim3d([1,1,Z,Y,X]) ->
    backward, against the same chain with the torch SSIM."""
    from gs_voxelizer_b200.losses import fused_ssim3d
    from gs_voxelizer_b200.optim_to_render import optim_to_render
    from gs_voxelizer_b200.voxelize import voxelize_gaussians
    from gs_voxelizer_b200.workloads import phantom
    cfg = K.small_config(vol=(48, 40, 56), n=3000, seed=97, scale=(0.005, 0.05))
    target = phantom(cfg, device="cuda")[..., 0]
    grads = []
    for ssim in (fused_ssim3d, torch_ssim3d):
        leaves = [torch.from_numpy(a).cuda().requires_grad_(True)
                  for a in K.inputs(cfg)]
        pr, cq, tmin, tmax, nt = optim_to_render(*leaves, cfg.vol, cfg.world,
                                                 cfg.center)
        vol = voxelize_gaussians(pr, cq, leaves[3], cfg.vol, tmin, tmax, nt)
        loss = ssim(vol.squeeze().unsqueeze(0).unsqueeze(0), target[None, None])
        loss.backward()
        grads.append([l.grad.clone() for l in leaves])
    for a, b, name in zip(*grads, ("pos3d", "scale3d", "quat", "intensity")):
        close(a.cpu().numpy(), b.cpu().numpy(), name)
