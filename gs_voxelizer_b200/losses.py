"""L1 loss against a target volume, standalone or fused into voxelization.

The reference leaves losses to its callers (FaCT-GS trains with L1 / SSIM in
PyTorch). These helpers compute the same L1 loss with this package's CUDA
kernels:

* ``l1_loss(vol, target)`` - drop-in for ``torch.nn.functional.l1_loss``
  (mean reduction by default): one reduction pass forward, one pass backward.
* ``voxelize_gaussians_l1(...)`` - voxelization with the loss fused in: the
  forward kernel reduces |vol - target| per tile while it stores the volume,
  and the backward kernel forms sign(vol - target) while it stages each tile,
  so dL/dvol is never materialised. Returns ``(loss, volume)``; gradients
  flow from the loss to the Gaussians (the volume output is not
  differentiable). With a ``SlabPlan`` it voxelizes one z-slab and, in the
  backward, all-reduces the per-Gaussian gradients over the process group.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
from torch.autograd import Function

from . import cuda as _C
from ._lib import check, i3, lib
from .slab import SlabPlan, allreduce_gaussian_grads, tile_layers


def _dev_check(t: torch.Tensor, name: str) -> None:
    _C._check_input(t, name)
    _C._check_f32(t, name)


class _L1Loss(Function):
    @staticmethod
    def forward(ctx, vol, target, denom):
        vol, target = vol.contiguous(), target.contiguous()
        _dev_check(vol, "vol")
        _dev_check(target, "target")
        if vol.shape != target.shape:
            raise ValueError(f"shape mismatch: {vol.shape} vs {target.shape}")
        n = vol.numel()
        loss = torch.empty((), dtype=torch.float32, device=vol.device)
        ws = _C._workspace(lib.gsv_l1_loss_workspace_bytes(n), vol.device)
        check(lib.gsv_l1_loss_forward(n, _C._ptr(vol), _C._ptr(target),
                                      float(denom), loss.data_ptr(),
                                      ws.data_ptr(), ws.numel(),
                                      _C._stream(vol.device)))
        ctx.denom = float(denom)
        ctx.save_for_backward(vol, target)
        return loss

    @staticmethod
    def backward(ctx, grad_loss):
        vol, target = ctx.saved_tensors
        grad_loss = grad_loss.contiguous().to(torch.float32)
        g = torch.empty_like(vol)
        check(lib.gsv_l1_loss_backward(vol.numel(), _C._ptr(vol),
                                       _C._ptr(target), grad_loss.data_ptr(),
                                       ctx.denom, _C._ptr(g),
                                       _C._stream(vol.device)))
        return g, None, None


def l1_loss(vol: torch.Tensor, target: torch.Tensor,
            reduction: str = "mean") -> torch.Tensor:
    """sum |vol - target| / numel ("mean") or the plain sum ("sum")."""
    if reduction not in ("mean", "sum"):
        raise ValueError(f"unsupported reduction {reduction!r}")
    denom = vol.numel() if reduction == "mean" else 1.0
    return _L1Loss.apply(vol, target, max(denom, 1))


class _VoxelizeL1(Function):
    @staticmethod
    def forward(ctx, pos3d_radii, conics, intensities, target, plan,
                tile_min, tile_max, denom, group, reduce):
        one_d = intensities.dim() == 1
        if one_d:
            intensities = intensities.unsqueeze(-1)
        C = _C._channels(intensities)
        for t, name in ((pos3d_radii, "pos3d_radii"), (conics, "conics"),
                        (intensities, "intensities"), (target, "target")):
            _dev_check(t, name)
        dev = pos3d_radii.device
        if tuple(target.shape) != (*plan.shape, C):
            raise ValueError(f"target shape {tuple(target.shape)} != "
                             f"{(*plan.shape, C)}")
        tile_min, tile_max = tile_min.contiguous(), tile_max.contiguous()
        n = int(pos3d_radii.shape[0])
        n_isect = plan.count(tile_min, tile_max)
        i32 = dict(dtype=torch.int32, device=dev)
        ids = torch.empty((n_isect,), **i32)
        bins = torch.empty((plan.num_tiles, 2), **i32)
        out = torch.empty(target.shape, dtype=torch.float32, device=dev)
        loss = torch.empty((), dtype=torch.float32, device=dev)
        ws = _C._workspace(lib.gsv_voxelize_l1_workspace_bytes(
            n, C, n_isect, i3(plan.vol), plan.tz0, plan.tz1), dev)
        # one call: binning, voxelization + loss, backward work plan in ws
        check(lib.gsv_voxelize_forward_l1(
            i3(plan.vol), plan.tz0, plan.tz1, C, n, n_isect,
            tile_min.data_ptr(), tile_max.data_ptr(), _C._ptr(pos3d_radii),
            _C._ptr(conics), _C._ptr(intensities), _C._ptr(target),
            float(denom), _C._ptr(ids), _C._ptr(bins), _C._ptr(out),
            loss.data_ptr(), None, None, ws.data_ptr(), ws.numel(),
            _C._stream(dev)))
        ctx.ws = ws
        ctx.plan, ctx.denom, ctx.group, ctx.one_d = plan, float(denom), group, one_d
        ctx.reduce = reduce
        ctx.save_for_backward(pos3d_radii, conics, intensities, ids, bins, out,
                              target)
        ctx.mark_non_differentiable(out)
        return loss, out

    @staticmethod
    def backward(ctx, grad_loss, _grad_out):
        pr, cq, inten, ids, bins, out, target = ctx.saved_tensors
        plan = ctx.plan
        C = inten.shape[1]
        n, n_isect, dev = int(pr.shape[0]), int(ids.numel()), pr.device
        f = dict(device=dev, dtype=torch.float32)
        gp = torch.empty((n, 4), **f)
        gc = torch.empty((n, 6), **f)
        gi = torch.empty((n, C), **f)
        if grad_loss is None:
            grad_loss = torch.zeros((), **f)
        grad_loss = grad_loss.contiguous().to(torch.float32)
        ws = ctx.ws  # records and work plan left by the forward
        check(lib.gsv_voxelize_backward_per_gaussian_l1(
            i3(plan.vol), plan.tz0, plan.tz1, C, n, n_isect, _C._ptr(ids),
            _C._ptr(bins), _C._ptr(pr), _C._ptr(cq), _C._ptr(inten),
            _C._ptr(out), _C._ptr(target), grad_loss.data_ptr(), ctx.denom,
            _C._ptr(gp), _C._ptr(gc), _C._ptr(gi), ws.data_ptr(), ws.numel(),
            _C._stream(dev)))
        if ctx.reduce:
            gp, gc, gi = allreduce_gaussian_grads([gp, gc, gi], ctx.group)
        if ctx.one_d:
            gi = gi.reshape(-1)
        return gp, gc, gi, None, None, None, None, None, None, None


def voxelize_gaussians_l1(
    pos3d_radii: torch.Tensor,
    conics: torch.Tensor,
    intensities: torch.Tensor,
    vol_size_voxel: Tuple[int, int, int],
    tile_min: torch.Tensor,
    tile_max: torch.Tensor,
    target: torch.Tensor,
    denom: Optional[float] = None,
    plan: Optional[SlabPlan] = None,
    group=None,
):
    """Voxelize and compute L = sum |vol - target| / denom in one pass.

    Args: as ``voxelize.voxelize_gaussians`` plus
        target: [Z,Y,X,C] float32 target (the slab's part with a plan).
        denom: normaliser; default the full volume's element count (mean).
        plan: SlabPlan for z-slab sharding; default the whole volume (then no
            collective, even inside a distributed job).
        group: process group for the gradient all-reduce (slab mode; default
            the default group when torch.distributed is initialised).
    Returns:
        (loss, volume): loss is a 0-d tensor (this slab's share with a plan),
        volume the forward volume (no gradient).
    """
    reduce = plan is not None
    if plan is None:
        plan = SlabPlan(vol_size_voxel, 0, tile_layers(vol_size_voxel))
    if denom is None:
        z, y, x = (int(v) for v in vol_size_voxel)
        C = 1 if intensities.dim() == 1 else int(intensities.shape[1])
        denom = float(z * y * x * C)
    return _VoxelizeL1.apply(pos3d_radii.contiguous(), conics.contiguous(),
                             intensities.contiguous(), target.contiguous(),
                             plan, tile_min.contiguous(),
                             tile_max.contiguous(), denom, group, reduce)


# ------------------------------------------------------------- 3D SSIM / TV

def _planar(t: torch.Tensor, name: str) -> Tuple[int, Tuple[int, int, int]]:
    """(channels, (D, H, W)) of a [..., D, H, W] volume: every leading
    dimension counts as a channel (the [B, C, D, H, W] layout of
    fused_ssim3d's callers, or [D, H, W])."""
    if t.dim() < 3:
        raise ValueError(f"{name} must have at least 3 dimensions (D, H, W)")
    d, h, w = (int(v) for v in t.shape[-3:])
    nch = 1
    for v in t.shape[:-3]:
        nch *= int(v)
    return nch, (d, h, w)


class _Ssim3d(Function):
    @staticmethod
    def forward(ctx, img1, img2, c1, c2):
        img1, img2 = img1.contiguous(), img2.contiguous()
        _dev_check(img1, "img1")
        _dev_check(img2, "img2")
        if img1.shape != img2.shape:
            raise ValueError(f"shape mismatch: {img1.shape} vs {img2.shape}")
        nch, dhw = _planar(img1, "img1")
        dims = i3(dhw)
        ws = _C._workspace(lib.gsv_ssim3d_workspace_bytes(nch, dims), img1.device)
        out = torch.empty((), dtype=torch.float32, device=img1.device)
        check(lib.gsv_ssim3d_forward(nch, dims, img1.data_ptr(), img2.data_ptr(),
                                     float(c1), float(c2), out.data_ptr(),
                                     ws.data_ptr(), ws.numel(),
                                     _C._stream(img1.device)))
        ctx.save_for_backward(img1, img2, ws)
        ctx.nch, ctx.dims = nch, dhw
        return out

    @staticmethod
    def backward(ctx, grad_out):
        img1, img2, ws = ctx.saved_tensors
        g = torch.empty_like(img1)
        grad_out = grad_out.contiguous().to(torch.float32)
        check(lib.gsv_ssim3d_backward(ctx.nch, i3(ctx.dims), img1.data_ptr(),
                                      img2.data_ptr(), grad_out.data_ptr(),
                                      ws.data_ptr(), ws.numel(), g.data_ptr(),
                                      _C._stream(img1.device)))
        return g, None, None, None


def fused_ssim3d(img1: torch.Tensor, img2: torch.Tensor,
                 c1: float = 0.01 ** 2, c2: float = 0.03 ** 2) -> torch.Tensor:
    """Mean 3D SSIM of img1 against img2 (Wang et al. 2004; 11^3 separable
    Gaussian window with sigma 1.5, zero padding), differentiable in img1.

    Volumes are [..., D, H, W] float32 CUDA tensors, every leading dimension
    a channel: the [B, C, D, H, W] call of the external fused_ssim3d in the
    reference's tests (test/test_gs_voxelizer.py:62) works unchanged, e.g.
    ``fused_ssim3d(vol.squeeze().unsqueeze(0).unsqueeze(0), target[None, None])``
    for a one-channel voxelizer output. Returns a 0-d tensor (higher is more
    similar; train with ``1 - fused_ssim3d(...)``)."""
    return _Ssim3d.apply(img1, img2, c1, c2)


class _Tv3d(Function):
    @staticmethod
    def forward(ctx, vol, isotropic, eps):
        vol = vol.contiguous()
        _dev_check(vol, "vol")
        nch, dhw = _planar(vol, "vol")
        dims = i3(dhw)
        ws = _C._workspace(lib.gsv_tv3d_workspace_bytes(nch, dims), vol.device)
        out = torch.empty((), dtype=torch.float32, device=vol.device)
        check(lib.gsv_tv3d(nch, dims, vol.data_ptr(), int(bool(isotropic)),
                           float(eps), out.data_ptr(), None, None, ws.data_ptr(),
                           ws.numel(), _C._stream(vol.device)))
        ctx.save_for_backward(vol, ws)
        ctx.nch, ctx.dims, ctx.iso, ctx.eps = nch, dhw, bool(isotropic), float(eps)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        vol, ws = ctx.saved_tensors
        g = torch.empty_like(vol)
        grad_out = grad_out.contiguous().to(torch.float32)
        check(lib.gsv_tv3d(ctx.nch, i3(ctx.dims), vol.data_ptr(), int(ctx.iso),
                           ctx.eps, None, grad_out.data_ptr(), g.data_ptr(),
                           ws.data_ptr(), ws.numel(), _C._stream(vol.device)))
        return g, None, None


def tv3d(vol: torch.Tensor, isotropic: bool = True, eps: float = 1e-8) -> torch.Tensor:
    """3D total variation of a [..., D, H, W] volume (leading dimensions are
    channels), mean over voxels and channels, with forward differences that
    are 0 across the far boundary: isotropic sqrt(dx^2 + dy^2 + dz^2 + eps)
    or anisotropic |dx| + |dy| + |dz|. Differentiable; a 0-d tensor."""
    if isotropic and not eps > 0:
        raise ValueError("isotropic TV needs eps > 0")
    return _Tv3d.apply(vol, isotropic, eps)
