"""bench.py's reference arm on the host cores (the one bench leg that needs no
GPU): one JSON line with the contract's keys, the same metric / unit / direction
as the GPU arm, rank 0 alone printing under torchrun. A small scene keeps it to
seconds."""

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench(*args, env=None):
    e = dict(os.environ)
    e.update(env or {})
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], cwd=ROOT, env=e,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    return [line for line in r.stdout.splitlines() if line.startswith("{")]


def test_reference_arm_json_line():
    import bench

    lines = _bench("--impl", "reference", "--n", "2000", "--steps", "1", "--warmup", "1")
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == bench.METRIC and d["unit"] == "MPix/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert d["steps"] == 1 and d["warmup"] == 1 and d["n_gpus"] == 1 and d["scaling"] == "weak"
    assert d["vs_baseline"] is None and d["dtype"] == "fp32" and "synthetic" in d["data"]
    assert d["config"]["workload"].startswith("config1") and d["config"]["gaussians_per_rank"] == 2000
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and "2000" in cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "MPix/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_prints_on_rank_0_only():
    assert _bench("--impl", "reference", "--n", "2000", "--steps", "1", "--warmup", "1",
                  env={"RANK": "1", "WORLD_SIZE": "2"}) == []


def test_config4_shards_and_cameras():
    """config 4 (the reference's multi-GPU configuration): every rank holds its own
    shard of the Gaussians and C / world of the 32 cameras; over the ranks the
    cameras are the one-rank set, in order, so the job's work is the same at any
    rank count (strong scaling)."""
    import torch

    import bench

    dev = torch.device("cpu")
    _, one = bench.make_params(800, 1, dev, 0, 1, "config4")
    assert one["viewmats"].shape == (32, 4, 4) and (one["width"], one["height"]) == (1600, 1200)
    for world in (2, 4, 8):
        parts = [bench.make_params(800 // world, 1 + r, dev, r, world, "config4") for r in range(world)]
        assert all(p["means"].shape[0] == 800 // world for p, _ in parts)
        assert torch.equal(torch.cat([d["viewmats"] for _, d in parts]), one["viewmats"])
        assert not torch.equal(parts[0][0]["means"], parts[1][0]["means"])


def test_reference_arm_samples_config1_only():
    lines = _bench("--impl", "reference", "--workload", "config4", "--steps", "1", "--warmup", "1")
    assert len(lines) == 1 and "unavailable" in json.loads(lines[0])


def test_clock_summary_window_and_reasons():
    """The clock record keeps the samples inside the timed window only, takes
    the median of the per-sample lowest SM clock over the job's GPUs and the
    union of the throttle reasons, which the bench line must report by name
    (hw_slowdown etc. make a run invalid)."""
    import bench

    s = bench.ClockSampler(["GPU-a", "GPU-b"])
    # (host time, lowest SM MHz over the GPUs, max MHz, highest watts, reasons bitmask)
    s.samples = [(0.5, 900.0, 1965.0, 100.0, 0x8),  # before the window: ignored
                 (1.0, 1965.0, 1965.0, 900.0, 0x0),
                 (1.1, 1900.0, 1965.0, 950.0, 0x4),
                 (1.2, 1965.0, 1965.0, 990.0, 0x0),
                 (3.0, 500.0, 1965.0, 100.0, 0x40)]  # after the window: ignored
    out = s.summary(1.0, 1.2)
    assert out["samples"] == 3 and out["gpus"] == 2
    assert out["sm_mhz"] == 1965.0 and out["sm_max_mhz"] == 1965.0
    assert out["power_w"] == 950.0
    assert out["reasons"] == ["sw_power_cap"]
    empty = bench.ClockSampler([])
    empty.__enter__()
    empty.__exit__(None, None, None)
    assert empty.summary(0.0, 1.0)["samples"] == 0
