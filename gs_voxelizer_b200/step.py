"""One training step of the path, sync-free, replayed as a CUDA graph.

The reference's step reads the pair count back to the host between the
projection and the binning (gs_voxelizer/voxelize.py:87-88) and allocates
its buffers per call (gs_voxelizer/cuda/bindings.cu:313-345, :670). Here one
step runs

    projection -> pair count -> binning -> voxelization with fused L1
    -> per-Gaussian backward -> projection backward

on one stream with no host read in between: the binning takes the capacity
of a persistent id buffer instead of the exact count. The count stays in
device memory; the loss and a flag "count > capacity" are copied to pinned
host memory at the end of the step, the only device->host transfer (8 bytes).
If the flag is set, the tile ranges were clamped to the capacity (nothing is
accessed out of bounds) and the results are invalid, so ``run()`` grows the
buffers and runs the step again before returning; growth is rare (the
capacity keeps 25 % headroom). Because the launch sequence and every
address are fixed, the whole step is captured once as a CUDA graph and
replayed: one graph launch per step instead of 14 kernel launches and the
Python around them.

With a process group of more than one rank (z-slab sharding), the step is
two graphs around one NCCL all-reduce of a flat buffer that holds the
per-Gaussian gradients, the slab's loss and its overflow flag, so every
rank sees the global loss and a global overflow decision.

Gradients are written to fixed tensors that are installed as the ``.grad``
of the parameter tensors; each step overwrites them (no accumulation).
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.distributed as dist

from . import cuda as _C
from ._lib import check, f3, i3, lib
from .slab import SlabPlan, tile_layers

_INT32_MAX = 2**31 - 1


class FusedL1Step:
    """L = sum |voxelize(Gaussians) - target| / denom and its gradients.

    Args:
        pos3d, scale3d, quat, intensities: the parameters (CUDA float32,
            contiguous, [N,3], [N,3], [N,4], [N,C] or [N]); the step reads
            them in place, so update them in place between steps.
        vol_size_voxel, vol_size_world, vol_center_pos: the volume, as for
            ``optim_to_render``.
        target: [Z,Y,X,C] float32 target of this rank's slab.
        denom: loss normaliser (default: element count of the full volume).
        plan: z-slab of this rank (default: the whole volume, no collective).
        group: process group whose ranks hold the other slabs (with a plan;
            default: the default group when torch.distributed is initialised).
        headroom: capacity of the pair buffer relative to the last count.
        use_graph: capture and replay CUDA graphs (False: launch eagerly).
    """

    def __init__(self, pos3d: torch.Tensor, scale3d: torch.Tensor,
                 quat: torch.Tensor, intensities: torch.Tensor,
                 vol_size_voxel: Tuple[int, int, int],
                 vol_size_world: Tuple[float, float, float],
                 vol_center_pos: Tuple[float, float, float],
                 target: torch.Tensor, denom: Optional[float] = None,
                 plan: Optional[SlabPlan] = None, group=None,
                 headroom: float = 1.25, use_graph: bool = True):
        self.params = (pos3d, scale3d, quat, intensities)
        for t, name in zip(self.params, ("pos3d", "scale3d", "quat", "intensities")):
            _C._check_input(t, name)
            _C._check_f32(t, name)
            if not t.is_contiguous():
                raise ValueError(f"{name} must be contiguous")
        self.n = int(pos3d.shape[0])
        if self.n < 1 or tuple(pos3d.shape) != (self.n, 3):
            raise ValueError(f"Invalid shape for pos3d: {tuple(pos3d.shape)}")
        if tuple(scale3d.shape) != (self.n, 3) or tuple(quat.shape) != (self.n, 4):
            raise ValueError("scale3d / quat shapes do not match pos3d")
        self.one_d = intensities.dim() == 1
        self.C = _C._channels(intensities)
        if intensities.shape[0] != self.n:
            raise ValueError("intensities do not match pos3d")
        self.vol = tuple(int(v) for v in vol_size_voxel)
        self.world = tuple(float(v) for v in vol_size_world)
        self.center = tuple(float(v) for v in vol_center_pos)
        self.plan = plan or SlabPlan(self.vol, 0, tile_layers(self.vol))
        if tuple(target.shape) != (*self.plan.shape, self.C):
            raise ValueError(f"target shape {tuple(target.shape)} != "
                             f"{(*self.plan.shape, self.C)}")
        _C._check_input(target, "target")
        _C._check_f32(target, "target")
        self.target = target.contiguous()
        if denom is None:
            z, y, x = self.vol
            denom = float(z * y * x * self.C)
        if denom == 0:
            raise ValueError("denom must be non-zero")
        self.denom = float(denom)
        self.group = group
        # only slabs are summed over ranks: a step over the whole volume is
        # complete on its own, even inside a distributed job
        self.ranks = (dist.get_world_size(group)
                      if plan is not None and dist.is_available()
                      and dist.is_initialized() else 1)
        if headroom < 1.0:
            raise ValueError("headroom must be >= 1")
        self.headroom = float(headroom)
        self.use_graph = bool(use_graph)
        self.device = pos3d.device

        n, C, dev = self.n, self.C, self.device
        f32 = dict(dtype=torch.float32, device=dev)
        i32 = dict(dtype=torch.int32, device=dev)
        self.pos3d_radii = torch.empty((n, 4), **f32)
        self.conics = torch.empty((n, 6), **f32)
        self.tile_min = torch.empty((n, 3), **i32)
        self.tile_max = torch.empty((n, 3), **i32)
        self.num_tiles_hit = torch.empty((n,), **i32)
        self.count = torch.zeros((1,), dtype=torch.int64, device=dev)
        # [pos3d_radii grad 4N | conics grad 6N | intensities grad CN | loss | overflow]
        self.flat = torch.zeros((n * (10 + C) + 2,), **f32)
        self.grad_pos3d_radii = self.flat[:4 * n].view(n, 4)
        self.grad_conics = self.flat[4 * n:10 * n].view(n, 6)
        self.grad_intensities = self.flat[10 * n:(10 + C) * n].view(n, C)
        self.loss = self.flat[(10 + C) * n:(10 + C) * n + 1]
        self.overflow = self.flat[(10 + C) * n + 1:]
        self.grad_loss = torch.ones((1,), **f32)
        self.grad_pos3d = torch.zeros((n, 3), **f32)
        self.grad_scale3d = torch.zeros((n, 3), **f32)
        self.grad_quat = torch.zeros((n, 4), **f32)
        self.volume = torch.empty((*self.plan.shape, C), **f32)
        self.bins = torch.empty((self.plan.num_tiles, 2), **i32)
        # (loss, overflow) read back once per step
        self._host = torch.zeros((2,), dtype=torch.float32).pin_memory()
        self.launches_per_step = 0
        self._vol_c, self._world_c, self._center_c = (
            i3(self.vol), f3(self.world), f3(self.center))
        self.capacity = 0
        self.ids = None
        self.ws = None
        self._graphs = None
        self.regrows = 0

        # size the pair buffer from one eager count
        self._project()
        self._count()
        self._resize(int(self.count.item()))

    # ---------------------------------------------------------------- stages

    def _stream(self) -> int:
        return _C._stream(self.device)

    def _project(self) -> None:
        pos, scale, quat, inten = self.params
        check(lib.gsv_optim_to_render_forward(
            self.n, self.C, pos.data_ptr(), scale.data_ptr(), quat.data_ptr(),
            inten.data_ptr(), self._vol_c, self._world_c, self._center_c,
            self.pos3d_radii.data_ptr(), self.conics.data_ptr(),
            self.tile_min.data_ptr(), self.tile_max.data_ptr(),
            self.num_tiles_hit.data_ptr(), self._stream()))

    def _count(self) -> None:
        check(lib.gsv_count_slab_intersects(
            self.n, self.tile_min.data_ptr(), self.tile_max.data_ptr(),
            self.plan.tz0, self.plan.tz1, self.count.data_ptr(),
            self._stream()))

    def _voxelize(self) -> None:
        p = self.plan
        inten = self.params[3]
        check(lib.gsv_voxelize_forward_l1(
            self._vol_c, p.tz0, p.tz1, self.C, self.n, self.capacity,
            self.tile_min.data_ptr(), self.tile_max.data_ptr(),
            self.pos3d_radii.data_ptr(), self.conics.data_ptr(),
            inten.data_ptr(), _C._ptr(self.target), self.denom,
            _C._ptr(self.ids), _C._ptr(self.bins), _C._ptr(self.volume),
            self.loss.data_ptr(), self.count.data_ptr(),
            self.overflow.data_ptr(), self.ws.data_ptr(), self.ws.numel(),
            self._stream()))
        check(lib.gsv_voxelize_backward_per_gaussian_l1(
            self._vol_c, p.tz0, p.tz1, self.C, self.n, self.capacity,
            _C._ptr(self.ids), _C._ptr(self.bins),
            self.pos3d_radii.data_ptr(), self.conics.data_ptr(),
            inten.data_ptr(), _C._ptr(self.volume), _C._ptr(self.target),
            self.grad_loss.data_ptr(), self.denom,
            self.grad_pos3d_radii.data_ptr(), self.grad_conics.data_ptr(),
            self.grad_intensities.data_ptr(), self.ws.data_ptr(),
            self.ws.numel(), self._stream()))

    def _project_backward(self) -> None:
        pos, scale, quat, _ = self.params
        check(lib.gsv_optim_to_render_backward(
            self.n, pos.data_ptr(), scale.data_ptr(), quat.data_ptr(),
            self._vol_c, self._world_c, self._center_c,
            self.grad_pos3d_radii.data_ptr(), self.grad_conics.data_ptr(),
            self.pos3d_radii.data_ptr(), self.grad_pos3d.data_ptr(),
            self.grad_scale3d.data_ptr(), self.grad_quat.data_ptr(),
            self._stream()))

    def _readback(self) -> None:
        self._host.copy_(self.flat[-2:], non_blocking=True)

    def _part_a(self) -> None:
        # the binning inside _voxelize writes the pair count and the
        # overflow flag (a float, so that the gradient all-reduce carries it)
        self._project()
        self._voxelize()

    def _part_b(self) -> None:
        self._project_backward()
        self._readback()

    def _allreduce(self) -> None:
        if self.ranks > 1:
            dist.all_reduce(self.flat, op=dist.ReduceOp.SUM, group=self.group)

    # -------------------------------------------------------------- capacity

    def _resize(self, count: int) -> None:
        cap = max(1024, int(count * self.headroom) + 1024)
        cap = min(cap, _INT32_MAX)
        if count > cap:
            raise RuntimeError(f"{count} (tile, gaussian) pairs exceed the "
                               f"int32 id range of one slab")
        self.capacity = cap
        dev = self.device
        self.ids = torch.empty((cap,), dtype=torch.int32, device=dev)
        p = self.plan
        nbytes = lib.gsv_voxelize_l1_workspace_bytes(
            self.n, self.C, cap, self._vol_c, p.tz0, p.tz1)
        self.ws = _C._workspace(nbytes, dev)
        self._graphs = None

    def _capture(self) -> None:
        # one eager pass first: lazy one-time setup (kernel attributes,
        # occupancy queries) happens outside the capture
        before = lib.gsv_launch_count()
        self._launch_eager()
        self.launches_per_step = int(lib.gsv_launch_count() - before)
        torch.cuda.current_stream(self.device).synchronize()
        ga, gb = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
        with torch.cuda.graph(ga):
            self._part_a()
        with torch.cuda.graph(gb):
            self._part_b()
        self._graphs = (ga, gb)

    # ------------------------------------------------------------------- run

    def _launch_eager(self) -> None:
        self._part_a()
        self._allreduce()
        self._part_b()

    def launch(self) -> None:
        """Queue one step on the current stream (no host synchronisation).
        Call ``finish()`` before using the loss or gradients."""
        if not self.use_graph:
            self._launch_eager()
            return
        if self._graphs is None:
            self._capture()
        ga, gb = self._graphs
        ga.replay()
        self._allreduce()
        gb.replay()

    def finish(self) -> bool:
        """Wait for the queued step; True if its results are valid (the
        pairs fitted the buffer), else the buffer has been grown and the step
        must be launched again."""
        torch.cuda.current_stream(self.device).synchronize()
        if self._host[1] == 0:
            return True
        # some rank overflowed: every rank grows (its own count) and repeats
        self.regrows += 1
        self._resize(max(int(self.count.item()), self.capacity))
        return False

    def run(self) -> float:
        """One step; returns the loss (the global loss with a process group)
        and leaves the gradients in the parameters' ``.grad``."""
        while True:
            self.launch()
            if self.finish():
                break
        self.install_grads()
        return float(self._host[0])

    def install_grads(self) -> None:
        pos, scale, quat, inten = self.params
        gi = self.grad_intensities.view(-1) if self.one_d else self.grad_intensities
        for t, g in ((pos, self.grad_pos3d), (scale, self.grad_scale3d),
                     (quat, self.grad_quat), (inten, gi)):
            if t.grad is not g:
                t.grad = g
