"""GPU tests of the owner-sharded step with halo exchange (halo.HaloL1Step).

Ranks are emulated by threads on one GPU with an in-process communicator
that implements the step's two collectives (all-gather of ints, all-to-all
of float buffers) with a barrier and device copies, so the whole protocol -
packing, exchange, unpacking, gradient return, accumulation, global loss and
overflow decision - runs on one GPU. The reference result is the single-GPU
fused step over the whole volume (step.FusedL1Step), which the other tests
tie to the oracle and to the reference. Tolerances: loss 1e-5 relative,
volume 1e-5 relative + 1e-6 absolute (summation order inside a tile
differs: owned Gaussians first, then the halo), gradients 1e-4 relative +
1e-4 of the array's max."""
import threading

import numpy as np
import pytest
import torch

from tests import _cases as K

pytestmark = pytest.mark.gpu


class _Shared:
    def __init__(self, world):
        self.world = world
        self.barrier = threading.Barrier(world, timeout=120)
        self.slots = [None] * world
        self.keep = {}  # symmetric buffers of all ranks, kept alive


class ThreadComm:
    """In-process stand-in for NcclComm: rank = thread."""

    def __init__(self, shared, rank):
        self.s, self.rank, self.world = shared, rank, shared.world

    def all_gather_ints(self, values, device):
        self.s.barrier.wait()
        self.s.slots[self.rank] = list(values)
        self.s.barrier.wait()
        out = [list(v) for v in self.s.slots]
        self.s.barrier.wait()
        return out

    def symmetric(self, key, numel, device):
        """p2p exchange: a buffer per rank, every rank's address known to all
        (on one GPU the 'peer' buffers are other threads' allocations)."""
        t = torch.zeros((numel,), dtype=torch.float32, device=device)
        torch.cuda.current_stream().synchronize()
        self.s.barrier.wait()
        self.s.slots[self.rank] = t
        self.s.barrier.wait()
        ptrs = [int(b.data_ptr()) for b in self.s.slots]
        self.s.keep.setdefault(key, {})[self.rank] = t
        self.s.barrier.wait()
        return t, ptrs

    def device_barrier(self, key):
        torch.cuda.current_stream().synchronize()
        self.s.barrier.wait()

    def all_to_all(self, send, send_counts, recv, recv_counts):
        torch.cuda.current_stream().synchronize()
        self.s.barrier.wait()
        self.s.slots[self.rank] = (send, list(send_counts))
        self.s.barrier.wait()
        off = 0
        for src in range(self.world):
            n = recv_counts[src]
            if n:
                ssend, scounts = self.s.slots[src]
                so = sum(scounts[:self.rank])
                assert scounts[self.rank] == n
                recv[off:off + n].copy_(ssend[so:so + n])
            off += n
        torch.cuda.current_stream().synchronize()
        self.s.barrier.wait()


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def close(got, want, rtol, atol_rel, name):
    got, want = got.double().cpu().numpy(), want.double().cpu().numpy()
    tol = rtol * np.abs(want) + atol_rel * max(np.abs(want).max(), 1e-30)
    bad = np.abs(got - want) > tol
    assert not bad.any(), f"{name}: {bad.sum()} of {bad.size} out of tolerance"


def _run_ranks(cfg, world, arrs, target_full, shrink=None, steps=2,
               exchange="nccl"):
    from gs_voxelizer_b200.halo import HaloL1Step, owner_of
    from gs_voxelizer_b200.slab import slab_bounds
    owners = owner_of(arrs[0], cfg.vol, cfg.world, cfg.center, world)
    shared = _Shared(world)
    results, errors = [None] * world, []

    def body(rank):
        try:
            torch.cuda.set_device(0)
            idx = np.nonzero(owners == rank)[0]
            params = [dev(a[idx]) for a in arrs]
            tz0, tz1 = slab_bounds(cfg.vol, world, rank)
            target = target_full[8 * tz0:min(cfg.vol[0], 8 * tz1)].contiguous()
            step = HaloL1Step(*params, cfg.vol, cfg.world, cfg.center, target,
                              comm=ThreadComm(shared, rank), use_graph=False,
                              exchange=exchange)
            if shrink is not None:  # every rank: `shrink` slots per peer,
                # too few, so the halo overflows
                step.caps_out = [0 if d == rank else shrink for d in range(world)]
                step.caps_in = [0 if d == rank else shrink for d in range(world)]
                step.caps_matrix = [[0 if a == b else shrink for b in range(world)]
                                    for a in range(world)]
                step._alloc_local()
                step._size_pairs(step.pair_cap)
            losses = [step.run() for _ in range(steps)]
            results[rank] = dict(idx=idx, losses=losses, step=step,
                                 grads=[p.grad.clone() for p in params],
                                 volume=step.volume.clone())
        except BaseException as exc:  # surface thread failures in the test
            errors.append(exc)
            shared.barrier.abort()

    threads = [threading.Thread(target=body, args=(r,)) for r in range(world)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=300)
    if errors:
        raise errors[0]
    return results


def _reference(cfg, arrs, target):
    from gs_voxelizer_b200.step import FusedL1Step
    params = [dev(a) for a in arrs]
    step = FusedL1Step(*params, cfg.vol, cfg.world, cfg.center, target)
    loss = step.run()
    return loss, [p.grad.clone() for p in params], step.volume.clone()


@pytest.mark.parametrize("exchange", ["nccl", "p2p"])
@pytest.mark.parametrize("world,channels", [(2, 1), (3, 1), (2, 3)])
def test_halo_step_matches_single_gpu(world, channels, exchange):
    from gs_voxelizer_b200.workloads import phantom
    from gs_voxelizer_b200.slab import slab_bounds
    cfg = K.small_config(vol=(72, 40, 48), n=4000, seed=80, channels=channels,
                         scale=(0.01, 0.06))
    arrs = list(K.inputs(cfg))
    target = phantom(cfg, device="cuda")
    want_loss, want_grads, want_vol = _reference(cfg, arrs, target)
    res = _run_ranks(cfg, world, arrs, target, exchange=exchange)
    halo = sum(sum(r["step"].caps_in) for r in res)
    assert halo > 0  # Gaussians do cross the slab boundaries
    for r in res:
        for l in r["losses"]:
            assert l == pytest.approx(want_loss, rel=1e-5)
        assert r["step"].regrows == 0
    # owned gradients, scattered back to global order
    for k, name in enumerate(("pos3d", "scale3d", "quat", "intensity")):
        got = torch.zeros_like(want_grads[k])
        for r in res:
            got[torch.from_numpy(r["idx"]).cuda()] = r["grads"][k]
        close(got, want_grads[k], 1e-4, 1e-4, name)
    for rank, r in enumerate(res):
        tz0, tz1 = slab_bounds(cfg.vol, world, rank)
        ref = want_vol[8 * tz0:min(cfg.vol[0], 8 * tz1)]
        err = (r["volume"].double() - ref.double()).abs()
        assert bool((err <= 1e-5 * ref.double().abs() + 1e-6).all()), float(err.max())


@pytest.mark.parametrize("exchange", ["nccl", "p2p"])
@pytest.mark.parametrize("slots", [1, 0])
def test_halo_overflow_regrows_on_every_rank(slots, exchange):
    """Too few halo slots: one per peer, or none at all (then no record
    slot exists and the overflow is known only from the senders' headers)."""
    from gs_voxelizer_b200.workloads import phantom
    cfg = K.small_config(vol=(64, 40, 40), n=3000, seed=81, scale=(0.01, 0.06))
    arrs = list(K.inputs(cfg))
    target = phantom(cfg, device="cuda")
    want_loss, want_grads, _ = _reference(cfg, arrs, target)
    res = _run_ranks(cfg, 2, arrs, target, shrink=slots, steps=1,
                     exchange=exchange)
    for r in res:
        assert r["step"].regrows == 1
        assert r["losses"][0] == pytest.approx(want_loss, rel=1e-5)
        assert max(r["step"].caps_out) > 1
    got = torch.zeros_like(want_grads[0])
    for r in res:
        got[torch.from_numpy(r["idx"]).cuda()] = r["grads"][0]
    close(got, want_grads[0], 1e-4, 1e-4, "pos3d")


def test_halo_single_rank_graph():
    """world = 1: no peers, the graph-replayed step equals FusedL1Step."""
    from gs_voxelizer_b200.halo import HaloL1Step
    from gs_voxelizer_b200.workloads import phantom

    class Solo:
        rank, world = 0, 1

    cfg = K.small_config(vol=(40, 36, 52), n=2000, seed=82, scale=(0.005, 0.05))
    arrs = list(K.inputs(cfg))
    target = phantom(cfg, device="cuda")
    want_loss, want_grads, want_vol = _reference(cfg, arrs, target)
    params = [dev(a) for a in arrs]
    step = HaloL1Step(*params, cfg.vol, cfg.world, cfg.center, target,
                      comm=Solo())
    for _ in range(2):
        assert step.run() == pytest.approx(want_loss, rel=1e-5)
    assert torch.equal(step.volume, want_vol)
    for p, g, name in zip(params, want_grads, ("pos3d", "scale3d", "quat", "intensity")):
        close(p.grad, g, 1e-4, 1e-4, name)


def test_halo_ranks_without_gaussians():
    """All Gaussians in the lowest slab of three: ranks 1 and 2 own none
    (rank 1 still receives rank 0's boundary Gaussians)."""
    from gs_voxelizer_b200.halo import owner_of
    from gs_voxelizer_b200.workloads import phantom
    cfg = K.small_config(vol=(72, 40, 48), n=2000, seed=83, pos=(0.0, 0.3),
                         scale=(0.01, 0.05))
    arrs = list(K.inputs(cfg))
    owners = owner_of(arrs[0], cfg.vol, cfg.world, cfg.center, 3)
    assert (owners == 2).sum() == 0
    target = phantom(cfg, device="cuda")
    want_loss, want_grads, _ = _reference(cfg, arrs, target)
    res = _run_ranks(cfg, 3, arrs, target, steps=1)
    for r in res:
        assert r["losses"][0] == pytest.approx(want_loss, rel=1e-5)
    assert res[2]["step"].n == 0
    got = torch.zeros_like(want_grads[0])
    for r in res:
        got[torch.from_numpy(r["idx"]).cuda()] = r["grads"][0]
    close(got, want_grads[0], 1e-4, 1e-4, "pos3d")
