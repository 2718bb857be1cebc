"""Multi-GPU tests over NCCL (skipped with fewer than two GPUs): the
owner-sharded halo step and the replicated step with a process group, each
rank a process on its own GPU, against the single-GPU step. Tolerances: loss
1e-5 relative; gradients 1e-4 of the array's max (summation order differs
across ranks)."""
import json
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_halo_and_replicated_steps_on_two_gpus(tmp_path):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
           "--master-port", str(_free_port()),
           os.path.join(ROOT, "tests", "multi", "halo_ranks.py"), str(tmp_path)]
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    for rank in range(2):
        res = json.load(open(tmp_path / f"rank{rank}.json"))
        want = res["ref_loss"]
        assert res["halo_slots_in"] > 0
        for loss in res["halo_loss"] + res["p2p_loss"] + res["rep_loss"]:
            assert loss == pytest.approx(want, rel=1e-5), res
        for e in res["halo_grad_err"] + res["p2p_grad_err"] + res["rep_grad_err"]:
            assert e < 1e-4, res
