"""Owner-sharded z-slab training step with a halo exchange (one process per GPU).

`step.FusedL1Step` with a process group replicates every Gaussian on every
rank: each rank projects all of them and one all-reduce sums all their
gradients, so that part of a step grows with the number of ranks. Here each
rank owns only a subset of the Gaussians (normally those whose centre lies
in its slab, see `owner_of`) and a step is

  A  project the owned Gaussians; pack the render records of those whose
     tile box reaches another rank's slab (`gsv_halo_pack`)
  -- exchange #1: records to the ranks that need them
  B  unpack the received halo after the owned Gaussians; voxelize the slab
     with the fused L1 loss and run the per-Gaussian backward over owned +
     halo; pack the halo's gradients, this rank's loss and overflow flags
  -- exchange #2: gradients back to their owners, plus every rank's header
  C  add the returned gradients to the owned ones in rank order; sum the
     ranks' losses in rank order; projection backward of the owned Gaussians

Traffic and per-rank work scale with the halo, not with the rank count, and
every rank ends a step with the global loss and a global overflow decision
without a further collective. An exchange is either two NCCL all-to-alls
(`exchange="nccl"`: A, B and C are three CUDA graphs with the collectives
between them) or direct writes of the packing kernels into the peers'
symmetric-memory receive buffers followed by this library's device barrier
(`exchange="p2p"`: the whole step is one CUDA graph). Segment capacities (halo slots per rank pair, the
pair buffer of the binning) keep 25 % headroom; an overflow anywhere makes
every rank re-size (one all-gather of the halo counts) and repeat the step.

Gradients of the owned parameters are written to fixed tensors installed as
their `.grad` (overwritten each step); the parameters are read in place.
Ownership is fixed when the step is built: a Gaussian that moves into
another rank's slab during training stays correct (it travels as halo every
step), only less efficient; rebuild the step with `owner_of` now and then
to re-balance.
"""
from __future__ import annotations

import ctypes
from typing import List, Optional, Sequence, Tuple

import numpy as np
import torch
import torch.distributed as dist

from . import cuda as _C
from ._lib import HALO_GRAD_FLOATS, HALO_RECORD_FLOATS, check, f3, i3, lib
from .slab import SlabPlan, slab_bounds, tile_layers

REC, GREC = HALO_RECORD_FLOATS, HALO_GRAD_FLOATS
_INT32_MAX = 2**31 - 1


def owner_of(pos3d: np.ndarray, vol_size_voxel, vol_size_world, vol_center_pos,
             world: int) -> np.ndarray:
    """Rank whose z-slab holds each Gaussian's centre (centres outside the
    volume go to the nearest slab). pos3d is [N, 3] (x, y, z) in world
    units; the volume tuples are (z, y, x) as for optim_to_render."""
    Z = int(vol_size_voxel[0])
    wz, cz = float(vol_size_world[0]), float(vol_center_pos[0])
    zv = (pos3d[:, 2].astype(np.float64) - (cz - 0.5 * wz)) / wz * Z
    tile = np.clip(np.floor(zv / 8.0), 0, tile_layers(vol_size_voxel) - 1).astype(np.int64)
    owners = np.empty(len(tile), dtype=np.int64)
    for r in range(world):
        tz0, tz1 = slab_bounds(vol_size_voxel, world, r)
        owners[(tile >= tz0) & (tile < tz1)] = r
    return owners


class NcclComm:
    """The two collectives the step needs, over a torch.distributed group."""

    def __init__(self, group=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)

    def all_gather_ints(self, values: Sequence[int], device) -> List[List[int]]:
        t = torch.tensor(list(values), dtype=torch.int64, device=device)
        out = [torch.empty_like(t) for _ in range(self.world)]
        dist.all_gather(out, t, group=self.group)
        return [o.tolist() for o in out]

    def all_to_all(self, send: torch.Tensor, send_counts: List[int],
                   recv: torch.Tensor, recv_counts: List[int]) -> None:
        dist.all_to_all_single(recv, send, recv_counts, send_counts,
                               group=self.group)


class SymmComm(NcclComm):
    """The step's exchanges as direct writes into the peers' receive buffers
    (torch symmetric memory over NVLink, plain stores from this library's
    packing kernels) followed by this library's device barrier across the
    ranks (gsv_peer_barrier, on a small symmetric signal array); the receive
    buffers are symmetric allocations of equal size on every rank. Nothing
    runs on the host between the stages, so a whole step can be one CUDA
    graph. NVLink multicast is not used (TORCH_SYMM_MEM_DISABLE_MULTICAST)."""

    graph_safe = True  # device_barrier is a graph-capturable kernel

    def __init__(self, group=None):
        super().__init__(group)
        import os
        os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
        self._handles = {}
        self._sig = None

    def _signals(self, device):
        if self._sig is None:
            import torch.distributed._symmetric_memory as symm_mem
            sig = symm_mem.empty(self.world, dtype=torch.int32, device=device)
            sig.zero_()
            torch.cuda.current_stream(device).synchronize()
            h = symm_mem.rendezvous(sig, self.group if self.group is not None
                                    else dist.group.WORLD)
            self._sig = (sig, h, _i64([int(p) for p in h.buffer_ptrs]),
                         torch.zeros((1,), dtype=torch.int32, device=device))
        return self._sig

    def symmetric(self, key: str, numel: int, device) -> Tuple[torch.Tensor, List[int]]:
        """A float32 buffer of numel elements on every rank (collective), and
        the device addresses of every rank's copy."""
        import torch.distributed._symmetric_memory as symm_mem
        t = symm_mem.empty(numel, dtype=torch.float32, device=device)
        t.zero_()
        # zeroed before any peer can write into it: the rendezvous below
        # returns on no rank before every rank has entered it
        torch.cuda.current_stream(device).synchronize()
        h = symm_mem.rendezvous(t, self.group if self.group is not None
                                else dist.group.WORLD)
        self._handles[key] = h
        return t, [int(p) for p in h.buffer_ptrs]

    def device_barrier(self, key: str) -> None:
        """Every rank's preceding writes into the buffers are visible to
        every rank after this point of its stream (one barrier kernel)."""
        sig, _, ptrs, epoch = self._signals(torch.device("cuda", torch.cuda.current_device()))
        check(lib.gsv_peer_barrier(self.world, self.rank, ptrs, epoch.data_ptr(),
                                   torch.cuda.current_stream().cuda_stream))


def segments(slots: Sequence[int], rank: int, rec: int) -> Tuple[List[int], List[int], int]:
    """Layout of an exchange buffer with one segment per peer: a header
    record plus slots[peer] record slots (none for the rank itself). Returns
    the element count of every segment (the all-to-all split sizes), the
    record offset of every segment and the total number of records."""
    counts, offs, off = [], [], 0
    for d, k in enumerate(slots):
        k = 0 if d == rank else int(k) + 1
        offs.append(off)
        counts.append(k * rec)
        off += k
    return counts, offs, off


def _i64(vals) -> ctypes.Array:
    return (ctypes.c_int64 * len(vals))(*[int(v) for v in vals])


def _i32(vals) -> ctypes.Array:
    return (ctypes.c_int32 * len(vals))(*[int(v) for v in vals])


class HaloL1Step:
    """L = sum |voxelize(all Gaussians) - target| / denom over all slabs,
    with this rank holding only its owned Gaussians.

    Args:
        pos3d, scale3d, quat, intensities: the OWNED parameters (CUDA
            float32, contiguous, [n,3], [n,3], [n,4], [n,C] or [n]).
        vol_size_voxel, vol_size_world, vol_center_pos: the whole volume.
        target: [Z_slab, Y, X, C] float32 target of this rank's slab.
        comm: collectives (default `NcclComm()` over the default group);
            rank r owns slab `slab_bounds(vol, world, r)`.
        denom: loss normaliser (default: element count of the whole volume).
        headroom: capacity of the buffers relative to the last counts.
        use_graph: capture stages A, B and C as CUDA graphs.
    """

    def __init__(self, pos3d, scale3d, quat, intensities, vol_size_voxel,
                 vol_size_world, vol_center_pos, target, comm=None,
                 denom: Optional[float] = None, headroom: float = 1.25,
                 use_graph: bool = True, exchange: str = "nccl"):
        if exchange not in ("nccl", "p2p"):
            raise ValueError("exchange must be 'nccl' or 'p2p'")
        self.comm = comm or (SymmComm() if exchange == "p2p" else NcclComm())
        self.p2p = exchange == "p2p"
        self.world, self.rank = self.comm.world, self.comm.rank
        if not 1 <= self.world <= 64:
            raise ValueError("1..64 ranks supported")
        self.params = (pos3d, scale3d, quat, intensities)
        for t, name in zip(self.params, ("pos3d", "scale3d", "quat", "intensities")):
            _C._check_input(t, name)
            _C._check_f32(t, name)
        self.n = int(pos3d.shape[0])
        if tuple(pos3d.shape) != (self.n, 3) or tuple(scale3d.shape) != (self.n, 3) \
                or tuple(quat.shape) != (self.n, 4) or intensities.shape[0] != self.n:
            raise ValueError("owned parameter shapes do not match")
        self.one_d = intensities.dim() == 1
        self.C = _C._channels(intensities)
        self.vol = tuple(int(v) for v in vol_size_voxel)
        self.wsize = tuple(float(v) for v in vol_size_world)
        self.center = tuple(float(v) for v in vol_center_pos)
        self.slabs = [slab_bounds(self.vol, self.world, r) for r in range(self.world)]
        self.plan = SlabPlan(self.vol, *self.slabs[self.rank])
        if tuple(target.shape) != (*self.plan.shape, self.C):
            raise ValueError(f"target shape {tuple(target.shape)} != "
                             f"{(*self.plan.shape, self.C)}")
        _C._check_input(target, "target")
        _C._check_f32(target, "target")
        self.target = target
        if denom is None:
            z, y, x = self.vol
            denom = float(z * y * x * self.C)
        if denom == 0:
            raise ValueError("denom must be non-zero")
        self.denom = float(denom)
        if headroom < 1.0:
            raise ValueError("headroom must be >= 1")
        self.headroom = float(headroom)
        self.use_graph = bool(use_graph)
        self.device = pos3d.device
        self._vol_c, self._world_c, self._center_c = (
            i3(self.vol), f3(self.wsize), f3(self.center))
        self._slab_tz = _i32([v for s in self.slabs for v in s])
        dev, n, C = self.device, self.n, self.C
        f32 = dict(dtype=torch.float32, device=dev)
        self.slot_map = torch.empty((max(n, 1), self.world), dtype=torch.int32, device=dev)
        self.halo_ws = _C._workspace(lib.gsv_halo_workspace_bytes(n, self.world), dev)
        self.halo_counts = torch.zeros((self.world,), dtype=torch.int64, device=dev)
        self.flags = torch.zeros((2,), **f32)   # pair overflow, halo overflow
        self.loss = torch.zeros((1,), **f32)
        self.count = torch.zeros((1,), dtype=torch.int64, device=dev)
        self.grad_loss = torch.ones((1,), **f32)
        self.out = torch.zeros((2,), **f32)     # global loss, global overflow
        self.grad_pos3d = torch.zeros((n, 3), **f32)
        self.grad_scale3d = torch.zeros((n, 3), **f32)
        self.grad_quat = torch.zeros((n, 4), **f32)
        self.volume = torch.empty((*self.plan.shape, C), **f32)
        self.bins = torch.empty((self.plan.num_tiles, 2), dtype=torch.int32, device=dev)
        self._host = torch.zeros((2,), dtype=torch.float32).pin_memory()
        self.regrows = 0
        self.launches_per_step = 0
        self._graphs = None
        self.caps_out = [0] * self.world   # slots this rank sends to each peer
        self.caps_in = [0] * self.world    # slots each peer sends to this rank
        self.caps_matrix = [[0] * self.world for _ in range(self.world)]
        self.n_loc = -1
        self.pair_cap = 0
        self.ids = None
        self.ws = None
        self._size_halo(initial=True)
        self._size_pairs()

    # -------------------------------------------------------------- layout

    def _alloc_local(self) -> None:
        """Local arrays: owned Gaussians first, then the halo slots of every
        peer in rank order; send / receive buffers of both exchanges."""
        n, C, dev = self.n, self.C, self.device
        self.n_loc = n + sum(self.caps_in)
        f32 = dict(dtype=torch.float32, device=dev)
        i32 = dict(dtype=torch.int32, device=dev)
        L = max(self.n_loc, 1)
        self.pr = torch.zeros((L, 4), **f32)
        self.cq = torch.zeros((L, 6), **f32)
        self.inten = torch.zeros((L, C), **f32)
        self.tmin = torch.zeros((L, 3), **i32)
        self.tmax = torch.zeros((L, 3), **i32)
        self.nt = torch.zeros((max(n, 1),), **i32)
        self.gp = torch.zeros((L, 4), **f32)
        self.gc = torch.zeros((L, 6), **f32)
        self.gi = torch.zeros((L, C), **f32)

        self.c1_send, self.o1_send, r1s = segments(self.caps_out, self.rank, REC)
        self.c1_recv, self.o1_recv, r1r = segments(self.caps_in, self.rank, REC)
        self.c2_send, self.o2_send, r2s = segments(self.caps_in, self.rank, GREC)
        self.c2_recv, self.o2_recv, r2r = segments(self.caps_out, self.rank, GREC)
        if self.p2p and self.world > 1:
            # symmetric receive buffers, equal sizes on every rank (the
            # largest any rank needs, from the all-gathered capacities);
            # each rank's packing kernels write its segments straight into
            # them (seg_dst), so there are no send buffers
            M = self.caps_matrix
            col = lambda d: [M[s][d] for s in range(self.world)]  # noqa: E731
            n1 = max(segments(col(d), d, REC)[2] for d in range(self.world))
            n2 = max(segments(M[d], d, GREC)[2] for d in range(self.world))
            self.recv1, p1 = self.comm.symmetric("recv1", max(n1, 1) * REC, dev)
            self.recv2, p2 = self.comm.symmetric("recv2", max(n2, 1) * GREC, dev)
            dst1 = [0] * self.world
            dst2 = [0] * self.world
            for d in range(self.world):
                if d == self.rank:
                    continue
                # this rank's segment in d's record buffer (laid out by the
                # slots every rank sends to d) and in d's gradient buffer
                # (laid out by the slots d sends to every rank)
                dst1[d] = p1[d] + 4 * REC * segments(col(d), d, REC)[1][self.rank]
                dst2[d] = p2[d] + 4 * GREC * segments(M[d], d, GREC)[1][self.rank]
            self._dst1, self._dst2 = _i64(dst1), _i64(dst2)
            self.send1 = self.send2 = None
        else:
            self.send1 = torch.zeros((max(r1s, 1) * REC,), **f32)
            self.recv1 = torch.zeros((max(r1r, 1) * REC,), **f32)
            self.send2 = torch.zeros((max(r2s, 1) * GREC,), **f32)
            self.recv2 = torch.zeros((max(r2r, 1) * GREC,), **f32)
        self._o1s, self._o1r = _i64(self.o1_send), _i64(self.o1_recv)
        self._o2s, self._o2r = _i64(self.o2_send), _i64(self.o2_recv)
        self._cap_out, self._cap_in = _i32(self.caps_out), _i32(self.caps_in)
        self._graphs = None

    def _size_halo(self, initial: bool = False) -> None:
        """Counts of owned Gaussians per peer -> all ranks agree on the
        segment capacities (one all-gather)."""
        if initial:
            self._alloc_local()  # zero-capacity segments: pack only counts
        self._project()
        self._pack()
        counts = self.halo_counts.tolist()
        caps = [0 if d == self.rank else
                int(c * self.headroom) + 16 if c > 0 else 0
                for d, c in enumerate(counts)]
        if not initial:  # never shrink: no oscillation between sizes
            caps = [max(c, o) for c, o in zip(caps, self.caps_out)]
        matrix = (self.comm.all_gather_ints(caps, self.device)
                  if self.world > 1 else [caps])
        caps_out = list(matrix[self.rank])
        caps_in = [matrix[s][self.rank] for s in range(self.world)]
        matrix = [list(r) for r in matrix]
        if matrix != self.caps_matrix:
            # (the same decision on every rank: the matrix is all-gathered)
            self.caps_matrix = matrix
            self.caps_out, self.caps_in = caps_out, caps_in
            self._alloc_local()

    def _size_pairs(self, count: Optional[int] = None) -> None:
        """Pair buffer of the binning from the local (owned + halo) set."""
        if count is None:
            self._project()
            self._pack()
            self.exchange_records()
            self._unpack()
            c = torch.zeros((1,), dtype=torch.int64, device=self.device)
            check(lib.gsv_count_slab_intersects(
                self.n_loc, self.tmin.data_ptr(), self.tmax.data_ptr(),
                self.plan.tz0, self.plan.tz1, c.data_ptr(), self._stream()))
            count = int(c.item())
        cap = min(max(1024, int(count * self.headroom) + 1024), _INT32_MAX)
        if count > cap:
            raise RuntimeError("more (tile, gaussian) pairs than int32 indices")
        cap = max(cap, self.pair_cap)
        if cap != self.pair_cap or self.ids is None:
            self.pair_cap = cap
            self.ids = torch.empty((cap,), dtype=torch.int32, device=self.device)
            self._graphs = None
        p = self.plan
        need = lib.gsv_voxelize_l1_workspace_bytes(
            max(self.n_loc, 0), self.C, cap, self._vol_c, p.tz0, p.tz1)
        if self.ws is None or self.ws.numel() < need:  # the local set grew
            self.ws = _C._workspace(need, self.device)
            self._graphs = None

    # -------------------------------------------------------------- stages

    def _stream(self) -> int:
        return _C._stream(self.device)

    def _project(self) -> None:
        pos, scale, quat, inten = self.params
        if self.n:
            check(lib.gsv_optim_to_render_forward(
                self.n, self.C, pos.data_ptr(), scale.data_ptr(),
                quat.data_ptr(), inten.data_ptr(), self._vol_c, self._world_c,
                self._center_c, self.pr.data_ptr(), self.cq.data_ptr(),
                self.tmin.data_ptr(), self.tmax.data_ptr(), self.nt.data_ptr(),
                self._stream()))
            self.inten[:self.n].copy_(inten.view(self.n, self.C))

    def _pack(self) -> None:
        args = (self.n, self.C, self.pr.data_ptr(), self.cq.data_ptr(),
                self.inten.data_ptr(), self.tmin.data_ptr(), self.tmax.data_ptr(),
                self.world, self.rank, self._slab_tz, _i64(self.o1_send),
                _i32(self.caps_out))
        tail = (self.slot_map.data_ptr(), self.halo_counts.data_ptr(),
                self.halo_ws.data_ptr(), self.halo_ws.numel(), self._stream())
        if self.send1 is None:
            check(lib.gsv_halo_pack_peers(*args, self._dst1, *tail))
        else:
            check(lib.gsv_halo_pack(*args, self.send1.data_ptr(), *tail))

    def _unpack(self) -> None:
        self.flags.zero_()
        check(lib.gsv_halo_unpack(
            self.n, self.C, self.world, self.rank, self._o1r, self._cap_in,
            self.recv1.data_ptr(), self.pr.data_ptr(), self.cq.data_ptr(),
            self.inten.data_ptr(), self.tmin.data_ptr(), self.tmax.data_ptr(),
            self.flags.data_ptr(), self._stream()))

    def stage_a(self) -> None:
        self._project()
        self._pack()

    def stage_b(self) -> None:
        self._unpack()
        p, n = self.plan, self.n_loc
        fl = self.flags
        check(lib.gsv_voxelize_forward_l1(
            self._vol_c, p.tz0, p.tz1, self.C, n, self.pair_cap,
            self.tmin.data_ptr(), self.tmax.data_ptr(), self.pr.data_ptr(),
            self.cq.data_ptr(), self.inten.data_ptr(), _C._ptr(self.target),
            self.denom, self.ids.data_ptr(), _C._ptr(self.bins),
            _C._ptr(self.volume), self.loss.data_ptr(), self.count.data_ptr(),
            fl[0:1].data_ptr(), self.ws.data_ptr(), self.ws.numel(),
            self._stream()))
        check(lib.gsv_voxelize_backward_per_gaussian_l1(
            self._vol_c, p.tz0, p.tz1, self.C, n, self.pair_cap,
            self.ids.data_ptr(), _C._ptr(self.bins), self.pr.data_ptr(),
            self.cq.data_ptr(), self.inten.data_ptr(), _C._ptr(self.volume),
            _C._ptr(self.target), self.grad_loss.data_ptr(), self.denom,
            self.gp.data_ptr(), self.gc.data_ptr(), self.gi.data_ptr(),
            self.ws.data_ptr(), self.ws.numel(), self._stream()))
        args = (self.n, self.C, self.world, self.rank, self._o2s, self._cap_in,
                self.gp.data_ptr(), self.gc.data_ptr(), self.gi.data_ptr(),
                self.loss.data_ptr(), self.flags.data_ptr())
        if self.send2 is None:
            check(lib.gsv_halo_pack_grads_peers(*args, self._dst2, self._stream()))
        else:
            check(lib.gsv_halo_pack_grads(*args, self.send2.data_ptr(),
                                          self._stream()))

    def stage_c(self) -> None:
        check(lib.gsv_halo_accumulate(
            self.n, self.C, self.world, self.rank, self._o2r,
            self.slot_map.data_ptr(), self.recv2.data_ptr(), self.gp.data_ptr(),
            self.gc.data_ptr(), self.gi.data_ptr(), self.loss.data_ptr(),
            self.flags.data_ptr(), self.out.data_ptr(), self._stream()))
        if self.n:
            pos, scale, quat, _ = self.params
            check(lib.gsv_optim_to_render_backward(
                self.n, pos.data_ptr(), scale.data_ptr(), quat.data_ptr(),
                self._vol_c, self._world_c, self._center_c, self.gp.data_ptr(),
                self.gc.data_ptr(), self.pr.data_ptr(),
                self.grad_pos3d.data_ptr(), self.grad_scale3d.data_ptr(),
                self.grad_quat.data_ptr(), self._stream()))
        self._host.copy_(self.out, non_blocking=True)

    def exchange_records(self) -> None:
        if self.world == 1:
            return
        if self.send1 is None:  # written in place by the peers' packing
            self.comm.device_barrier("recv1")
        else:
            self.comm.all_to_all(self.send1, self.c1_send, self.recv1,
                                 self.c1_recv)

    def exchange_grads(self) -> None:
        if self.world == 1:
            return
        if self.send2 is None:
            self.comm.device_barrier("recv2")
        else:
            self.comm.all_to_all(self.send2, self.c2_send, self.recv2,
                                 self.c2_recv)

    # ---------------------------------------------------------------- run

    def _whole_step(self) -> None:
        self.stage_a()
        self.exchange_records()
        self.stage_b()
        self.exchange_grads()
        self.stage_c()

    def _capture(self) -> None:
        before = lib.gsv_launch_count()
        self._whole_step()
        self.launches_per_step = int(lib.gsv_launch_count() - before)
        torch.cuda.current_stream(self.device).synchronize()
        if self.world == 1 or getattr(self.comm, "graph_safe", False):
            # exchanges by device barriers (or none): the whole step is one
            # graph
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self._whole_step()
            self._graphs = [g]
            return
        graphs = []
        for stage in (self.stage_a, self.stage_b, self.stage_c):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                stage()
            graphs.append(g)
        self._graphs = graphs

    def launch(self) -> None:
        """Queue one step (A, exchange, B, exchange, C) on the current
        stream; `finish()` waits for it."""
        if not self.use_graph:
            self.stage_a()
            self.exchange_records()
            self.stage_b()
            self.exchange_grads()
            self.stage_c()
            return
        if self._graphs is None:
            self._capture()
        if len(self._graphs) == 1:
            self._graphs[0].replay()
            return
        ga, gb, gc = self._graphs
        ga.replay()
        self.exchange_records()
        gb.replay()
        self.exchange_grads()
        gc.replay()

    def finish(self) -> bool:
        """Wait for the queued step; True if valid on every rank, else the
        buffers have been re-sized on every rank (collectively) and the step
        must be launched again."""
        torch.cuda.current_stream(self.device).synchronize()
        if self._host[1] == 0:
            return True
        self.regrows += 1
        own = int(self.count.item())
        self._size_halo()
        self._size_pairs(max(own, self.pair_cap))
        self._graphs = None
        return False

    def run(self) -> float:
        """One step; returns the global loss and leaves the owned
        parameters' gradients in their `.grad`."""
        while True:
            self.launch()
            if self.finish():
                break
        self.install_grads()
        return float(self._host[0])

    def install_grads(self) -> None:
        pos, scale, quat, inten = self.params
        gi = self.gi[:self.n]
        if self.one_d:
            gi = gi.view(-1)
        for t, g in ((pos, self.grad_pos3d), (scale, self.grad_scale3d),
                     (quat, self.grad_quat), (inten, gi)):
            if t.grad is not g:
                t.grad = g
