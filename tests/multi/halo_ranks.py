"""Run by tests/test_gpu_multi.py under torch.distributed.run (one process
per GPU, NCCL): the owner-sharded step (halo.HaloL1Step, with NCCL
all-to-alls and with direct peer writes + device barriers) and the replicated
step (step.FusedL1Step with a process group) against the single-GPU step
over the whole volume, computed on every rank. Writes one JSON result per
rank into the directory given as argv[1]."""
import json
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", ".."))

from gs_voxelizer_b200.halo import HaloL1Step, owner_of  # noqa: E402
from gs_voxelizer_b200.slab import SlabPlan, slab_bounds  # noqa: E402
from gs_voxelizer_b200.step import FusedL1Step  # noqa: E402
from gs_voxelizer_b200.workloads import phantom  # noqa: E402
from tests import _cases as K  # noqa: E402


def rel_err(a, b):
    a, b = a.double(), b.double()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


def main():
    out_dir = sys.argv[1]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("nccl", device_id=torch.device("cuda", int(os.environ["LOCAL_RANK"])))
    cfg = K.small_config(vol=(96, 48, 56), n=6000, seed=90, scale=(0.01, 0.06))
    arrs = list(K.inputs(cfg))
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    target = phantom(cfg, device="cuda")
    # single-GPU reference, on every rank
    ref_params = [dev(a) for a in arrs]
    ref = FusedL1Step(*ref_params, cfg.vol, cfg.world, cfg.center, target)
    ref_loss = ref.run()
    ref_grads = [p.grad.clone() for p in ref_params]
    tz0, tz1 = slab_bounds(cfg.vol, world, rank)
    slab_target = target[8 * tz0:min(cfg.vol[0], 8 * tz1)].contiguous()
    res = {"rank": rank, "ref_loss": ref_loss}
    # owner-sharded
    owners = owner_of(arrs[0], cfg.vol, cfg.world, cfg.center, world)
    idx = np.nonzero(owners == rank)[0]
    own = [dev(a[idx]) for a in arrs]
    halo = HaloL1Step(*own, cfg.vol, cfg.world, cfg.center, slab_target)
    res["halo_loss"] = [halo.run() for _ in range(3)]
    res["halo_slots_in"] = sum(halo.caps_in)
    ii = torch.from_numpy(idx).cuda()
    res["halo_grad_err"] = [rel_err(p.grad, g[ii]) for p, g in zip(own, ref_grads)]
    # owner-sharded, exchanges as direct writes into the peers' symmetric
    # receive buffers + device barriers
    own2 = [dev(a[idx]) for a in arrs]
    halo2 = HaloL1Step(*own2, cfg.vol, cfg.world, cfg.center, slab_target,
                       exchange="p2p")
    res["p2p_loss"] = [halo2.run() for _ in range(3)]
    res["p2p_grad_err"] = [rel_err(p.grad, g[ii]) for p, g in zip(own2, ref_grads)]
    del halo2
    # replicated
    rep_params = [dev(a) for a in arrs]
    rep = FusedL1Step(*rep_params, cfg.vol, cfg.world, cfg.center, slab_target,
                      denom=float(np.prod(cfg.vol)), plan=SlabPlan(cfg.vol, tz0, tz1))
    res["rep_loss"] = [rep.run() for _ in range(2)]
    res["rep_grad_err"] = [rel_err(p.grad, g) for p, g in zip(rep_params, ref_grads)]
    with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
        json.dump(res, f)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
