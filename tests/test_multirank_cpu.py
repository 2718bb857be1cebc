"""Multi-rank host logic of the z-slab sharding on CPU with the gloo backend
(world_size 2, 127.0.0.1). Each rank runs the oracle on its slab; the
per-Gaussian gradients are summed with the package's all-reduce helper and
must equal the single-process gradients. Also checks that a rank that fails
before the collective surfaces as an error on the other rank (short
process-group timeout), not as a hang."""
import os
import socket
import traceback
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _init(rank, world, port, timeout_s=60):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=timedelta(seconds=timeout_s))


def _case():
    from tests import _cases as K
    cfg = K.small_config(vol=(56, 24, 32), n=400, seed=60, scale=(0.01, 0.06))
    return cfg


def _sharded_worker(rank, world, port, out_path):
    try:
        import sys
        sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        from gs_voxelizer_b200.slab import allreduce_gaussian_grads, slab_bounds
        from oracle import oracle as O
        from tests import _cases as K
        _init(rank, world, port)
        cfg = _case()
        pos, scale, quat, inten = K.inputs(cfg)
        pr, cq, tmin, tmax, nt = O.optim_to_render_forward(
            pos, scale, quat, inten, cfg.vol, cfg.world, cfg.center)
        tz0, tz1 = slab_bounds(cfg.vol, world, rank)
        z0, z1 = 8 * tz0, min(cfg.vol[0], 8 * tz1)
        rng = np.random.default_rng(7)
        W = rng.standard_normal((*cfg.vol, 1)).astype(np.float32)
        gp, gc, gi = O.voxelize_backward(cfg.vol, tmin, tmax, pr, cq, inten,
                                         W[z0:z1], tile_z=(tz0, tz1))
        ids, bins = O.bin_and_sort_gaussians(tmin, tmax, cfg.vol, tile_z=(tz0, tz1))
        vol = O.voxelize_forward(cfg.vol, ids, bins, pr, cq, inten, tile_z=(tz0, tz1))
        partial = torch.tensor([float((vol.astype(np.float64) * W[z0:z1]).sum())],
                               dtype=torch.float64)
        dist.all_reduce(partial)
        grads = allreduce_gaussian_grads([torch.from_numpy(g) for g in (gp, gc, gi)])
        if rank == 0:
            np.savez(out_path, gp=grads[0].numpy(), gc=grads[1].numpy(),
                     gi=grads[2].numpy(), loss=partial.numpy())
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        traceback.print_exc()
        raise


def test_sharded_gradients_equal_single_process(tmp_path):
    from oracle import oracle as O
    from tests import _cases as K
    world, port = 2, _free_port()
    out = str(tmp_path / "r0.npz")
    mp.start_processes(_sharded_worker, args=(world, port, out), nprocs=world,
                       start_method="spawn")
    got = np.load(out)
    cfg = _case()
    pos, scale, quat, inten = K.inputs(cfg)
    pr, cq, tmin, tmax, nt = O.optim_to_render_forward(
        pos, scale, quat, inten, cfg.vol, cfg.world, cfg.center)
    rng = np.random.default_rng(7)
    W = rng.standard_normal((*cfg.vol, 1)).astype(np.float32)
    gp, gc, gi = O.voxelize_backward(cfg.vol, tmin, tmax, pr, cq, inten, W)
    ids, bins = O.bin_and_sort_gaussians(tmin, tmax, cfg.vol)
    vol = O.voxelize_forward(cfg.vol, ids, bins, pr, cq, inten)
    assert got["loss"][0] == pytest.approx(float((vol.astype(np.float64) * W).sum()), rel=1e-9)
    for a, b in ((got["gp"], gp), (got["gc"], gc), (got["gi"], gi)):
        tol = 1e-4 * np.abs(b) + 1e-5 * np.abs(b).max()
        assert (np.abs(a - b) <= tol).all()


def _failing_worker(rank, world, port, out_path):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    _init(rank, world, port, timeout_s=5)
    if rank == 1:
        # this rank fails between steps, before joining the all-reduce
        os._exit(3)
    from gs_voxelizer_b200.slab import allreduce_gaussian_grads
    status = "hung"
    try:
        allreduce_gaussian_grads([torch.ones(4), torch.ones(6)])
        status = "completed"
    except Exception as exc:  # the peer never joins: gloo reports an error
        status = "error:" + type(exc).__name__
    with open(out_path, "w") as f:
        f.write(status)
    os._exit(0)


def test_rank_failure_surfaces_as_error(tmp_path):
    world, port = 2, _free_port()
    out = str(tmp_path / "status.txt")
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_failing_worker, args=(r, world, port, out))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert os.path.exists(out)
    assert open(out).read().startswith("error:")


def test_owner_of_assigns_each_centre_to_its_slab():
    """halo.owner_of: the rank whose z-slab holds each Gaussian's centre,
    consistent with slab_bounds; centres outside the volume go to the
    nearest slab."""
    from gs_voxelizer_b200.halo import owner_of
    from gs_voxelizer_b200.slab import slab_bounds
    vol, world_size, center = (100, 30, 20), (2.0, 1.0, 1.0), (1.0, 0.5, 0.5)
    rng = np.random.default_rng(0)
    pos = rng.uniform(-0.2, 2.2, size=(5000, 3)).astype(np.float32)
    for world in (1, 2, 3, 5):
        own = owner_of(pos, vol, world_size, center, world)
        assert own.min() >= 0 and own.max() < world
        zv = pos[:, 2].astype(np.float64) / 2.0 * 100  # volume starts at z = 0
        tile = np.clip(np.floor(zv / 8), 0, 12)
        for r in range(world):
            tz0, tz1 = slab_bounds(vol, world, r)
            assert ((tile >= tz0) & (tile < tz1) == (own == r)).all()


def _halo_layout_worker(rank, world, port):
    try:
        import sys
        sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        from gs_voxelizer_b200.halo import REC, NcclComm, segments
        _init(rank, world, port)
        comm = NcclComm()
        # slots this rank sends to every peer; everyone learns the matrix
        mine = [0 if d == rank else 3 * (rank + 1) + d for d in range(world)]
        matrix = comm.all_gather_ints(mine, "cpu")
        caps_out = matrix[rank]
        caps_in = [matrix[s][rank] for s in range(world)]
        c_send, o_send, n_send = segments(caps_out, rank, REC)
        c_recv, o_recv, n_recv = segments(caps_in, rank, REC)
        send = torch.full((n_send * REC,), -1.0)
        recv = torch.full((n_recv * REC,), -2.0)
        for d in range(world):
            for slot in range(caps_out[d] + 1 if d != rank else 0):
                r = (o_send[d] + slot) * REC
                send[r:r + 3] = torch.tensor([rank, d, slot], dtype=torch.float32)
        comm.all_to_all(send, c_send, recv, c_recv)
        for s in range(world):
            for slot in range(caps_in[s] + 1 if s != rank else 0):
                r = (o_recv[s] + slot) * REC
                assert recv[r:r + 3].tolist() == [s, rank, slot], (rank, s, slot)
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        traceback.print_exc()
        raise


def test_halo_exchange_layout_over_gloo():
    """halo.segments + the communicator: every rank's send segments land
    in the peers' receive segments slot for slot (header included), with
    capacities agreed through the all-gather (3 gloo ranks)."""
    mp.spawn(_halo_layout_worker, args=(3, _free_port()), nprocs=3, join=True)
