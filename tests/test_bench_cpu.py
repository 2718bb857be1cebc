"""Host-side helpers of bench.py that need no GPU."""
import importlib.util
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    spec = importlib.util.spec_from_file_location("bench", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_clock_samples_report_throttle_reasons():
    b = _bench()
    text = "\n".join([
        "0, 1965, 1965, 650.1, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active",
        "0, 1950, 1965, 910.3, 0x0000000000000004, Not Active, Not Active, Not Active, Active",
        "0, 1800, 1965, 990.0, 0x0000000000000008, Active, Not Active, Not Active, Active",
        "garbage line",
    ])
    c = b.parse_clock_samples(text)
    assert c["samples"] == 3 and c["sm_mhz"] == 1950 and c["sm_max_mhz"] == 1965
    assert c["reasons"] == ["hw_slowdown", "sw_power_cap"]
    assert b.parse_clock_samples("") is None


def test_weak_workload_and_inputs_scale_with_ranks():
    """The N-rank workload stacks N 256-deep slabs with N x 100k Gaussians
    whose centres cover the whole stacked depth."""
    b = _bench()
    cfg = b.workload(4)
    assert cfg.vol == (1024, 256, 256) and cfg.n == 400_000
    pos, scale, quat, inten = b.make_inputs(cfg, 4)
    zv = (pos[:, 2] - (cfg.center[0] - 0.5 * cfg.world[0])) / cfg.world[0]
    hist = np.histogram(zv, bins=4, range=(0.0, 1.0))[0]
    assert hist.min() > 0.2 * len(zv)  # every slab gets about a quarter


def test_hbm_roofline_uses_measured_peak(tmp_path):
    b = _bench()
    peaks = tmp_path / "peaks.json"
    peaks.write_text('{"hbm_gbs": 6558.7}')
    r = b.hbm_roofline("backward", 0.304, 256 ** 3, 158619648, str(peaks))
    assert r["bound"] == "hbm" and r["unit"] == "GB/s" and r["peak"] == 6558.7
    assert r["algorithmic_bytes"] == 8 * 256 ** 3
    assert abs(r["achieved"] - 8 * 256 ** 3 / 0.304e-3 / 1e9) < 1e-6
    assert abs(r["frac"] - r["achieved"] / 6558.7) < 1e-12
    assert r["peak_source"] == "measured hbm_gbs"
    r = b.hbm_roofline("forward", 0.18, 100, None, str(tmp_path / "missing.json"))
    assert r["peak"] == b.FALLBACK_HBM_GBS and r["peak_source"] == "fallback hbm_gbs"


def test_halo_step_falls_back_to_nccl(monkeypatch):
    """bench.make_halo_step: the p2p exchange when it can be set up, else the
    NCCL exchange, and EXCHANGE_USED says which (no GPU: a stand-in class)."""
    import bench

    class Step:
        def __init__(self, *args, exchange, **kw):
            if exchange == "p2p" and Step.fail:
                raise RuntimeError("no symmetric memory")
            self.exchange, self.kw = exchange, kw

    class Cfg:
        vol, world, center = (8, 8, 8), (1.0, 1.0, 1.0), (0.5, 0.5, 0.5)

    monkeypatch.setattr(bench, "EXCHANGE", "p2p")
    Step.fail = False
    s = bench.make_halo_step(Step, [1, 2, 3, 4], Cfg, "t", denom=3.0)
    assert s.exchange == "p2p" and bench.EXCHANGE_USED == "p2p" and s.kw == {"denom": 3.0}
    Step.fail = True
    s = bench.make_halo_step(Step, [1, 2, 3, 4], Cfg, "t")
    assert s.exchange == "nccl" and bench.EXCHANGE_USED == "nccl"
    monkeypatch.setattr(bench, "EXCHANGE", "nccl")
    Step.fail = False
    assert bench.make_halo_step(Step, [1, 2, 3, 4], Cfg, "t").exchange == "nccl"
