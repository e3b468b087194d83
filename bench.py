"""Benchmark of the 3DGS training hot path: rasterization() forward + backward +
SelectiveAdam.step, on BASELINE config 1 (1M Gaussians, one 1297x840 pinhole
camera, fx=fy=1150, SH degree 3, packed=True, fp32).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl gsb|reference]

Prints ONE JSON line (rank 0). ``value`` is whole-job MPix/s (rendered pixels per
second over all ranks, fwd+bwd+Adam per pixel batch); ``ms_per_step`` is the
fwd+bwd+Adam time of one step. With N>1 (torchrun) every rank owns its own 1M
Gaussian shard and one camera, and rasterization(distributed=True) exchanges the
projected splats with NCCL all-to-all (weak scaling: fixed work per GPU).

``--impl reference`` times the CPU restatement of the reference algorithm
(oracle/, the reference's CUDA extension cannot be built here) on the host cores,
on a bounded sample of the same step.
"""

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "fwd+bwd+Adam ms/iter at 1M Gaussians 1297x840; MPix/s at 1/2/4/8 GPUs"
GRAD_BANK = 4
WORKLOADS = {
    "config1": "config1: 1M Gaussians, 1297x840 pinhole fx=fy=1150, SH deg 3, packed, fwd+bwd+SelectiveAdam",
    "config3": ("config3: 3M Gaussians, 8 cameras 1920x1080 fx=fy=1500 on a radius-8 sphere, SH deg 3, "
                "packed, fwd+bwd+SelectiveAdam"),
    "config4": ("config4: 6M Gaussians sharded over the ranks, 32 cameras 1600x1200 fx=fy=1200 on a radius-8 "
                "sphere split over the ranks, SH deg 3, packed, fwd+bwd+SelectiveAdam"),
    "config2": ("config2: 500k Gaussians, 4 cameras 1024x1024 fx=fy=1024 on a radius-6 ring, SH deg 3, RGB+ED, "
                "antialiased, absgrad, packed, fwd+bwd"),
}
# rasterization() options and whether the step ends with the optimizer, per workload
STEP_MODES = {
    "config1": dict(render_mode="RGB", rasterize_mode="classic", absgrad=False, adam=True),
    "config3": dict(render_mode="RGB", rasterize_mode="classic", absgrad=False, adam=True),
    "config4": dict(render_mode="RGB", rasterize_mode="classic", absgrad=False, adam=True),
    "config2": dict(render_mode="RGB+ED", rasterize_mode="antialiased", absgrad=True, adam=False),
}
LRS = {"means": 1.6e-4, "scales": 5e-3, "quats": 1e-3, "opacities": 5e-2, "sh": 2.5e-3}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="gsb", choices=["gsb", "reference"])
    ap.add_argument("--n", type=int, default=None, help="Gaussians per rank (default: the workload's)")
    ap.add_argument("--workload", default="config1", choices=["config1", "config2", "config3", "config4"],
                    help="config1 (the headline, default), config2 (500k Gaussians, 4 cameras at "
                         "1024x1024, RGB+ED, antialiased, absgrad, fwd+bwd), config3 (3M Gaussians, 8 "
                         "cameras at 1920x1080) or config4 (6M Gaussians sharded over the ranks, 32 "
                         "cameras at 1600x1200 split over the ranks: total work fixed)")
    ap.add_argument("--dense", action="store_true",
                    help="rasterization(packed=False), the reference trainer's default layout")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-sharded", action="store_true",
                    help="skip the sharded config-4 measurement reported under 'sharded'")
    ap.add_argument("--profile-ops", action="store_true", help="print per-op breakdown to stderr")
    return ap.parse_args()


# Child process that reads the GPU's SM clock, power and clock-event reasons
# through NVML (the library nvidia-smi queries) every PERIOD seconds and prints
# one timestamped line per sample. A separate process keeps the sampling off the
# benchmark's Python thread. Only reads: it changes no setting.
_SAMPLER_CHILD = r"""
import sys, time
import pynvml as N
N.nvmlInit()
keys, period = sys.argv[1].split(";"), float(sys.argv[2])
hs = [N.nvmlDeviceGetHandleByUUID(k) if k.startswith("GPU-") else N.nvmlDeviceGetHandleByIndex(int(k))
      for k in keys]
mx = min(N.nvmlDeviceGetMaxClockInfo(h, N.NVML_CLOCK_SM) for h in hs)
reasons = getattr(N, "nvmlDeviceGetCurrentClocksEventReasons", None) or N.nvmlDeviceGetCurrentClocksThrottleReasons
while True:
    # one line per tick over all the job's GPUs: the lowest SM clock, the
    # highest power draw and the union of the active reasons
    t = time.time()
    sm = min(N.nvmlDeviceGetClockInfo(h, N.NVML_CLOCK_SM) for h in hs)
    r = 0
    for h in hs:
        r |= reasons(h)
    p = max(N.nvmlDeviceGetPowerUsage(h) for h in hs) / 1000.0
    sys.stdout.write(f"{t:.4f},{sm},{mx},{p:.1f},{r}\n")
    sys.stdout.flush()
    time.sleep(period)
"""

# NVML clock-event reason bits (nvml.h) with nvidia-smi's names
_REASON_BITS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
                0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}


def gpu_key(device):
    """NVML key of a CUDA device: its UUID, else its index."""
    import torch

    props = torch.cuda.get_device_properties(device)
    uuid = str(getattr(props, "uuid", ""))
    return uuid if uuid.startswith("GPU-") else ("GPU-" + uuid if uuid else str(device.index or 0))


class ClockSampler:
    """Samples SM clocks and clock-event (throttle) reasons while the benchmark
    runs: started before the warm-up, confirmed running (first sample received)
    before returning, and summarised over the samples taken inside a given host
    time window (the timed region). One child process samples all the given
    GPUs (rank 0 samples the whole job's; the other ranks start none, which keeps
    the host cores for the ranks' own work)."""

    PERIOD = 0.01

    def __init__(self, keys):
        self.keys = list(keys)
        self.samples = []  # (time, lowest sm_mhz, max_mhz, highest watts, reasons bitmask)
        self.proc = None
        self.error = None

    def __enter__(self):
        if not self.keys:
            return self
        try:
            self.proc = subprocess.Popen([sys.executable, "-c", _SAMPLER_CHILD, ";".join(self.keys),
                                          str(self.PERIOD)],
                                         stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)
        except OSError as e:
            self.error = str(e)
            return self
        self.ready = threading.Event()
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()
        if not self.ready.wait(timeout=30):
            self.error = "no sample within 30 s"
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = line.strip().split(",")
            if len(parts) == 5:
                try:
                    self.samples.append((float(parts[0]), float(parts[1]), float(parts[2]), float(parts[3]),
                                         int(parts[4])))
                except ValueError:
                    continue
                self.ready.set()
        self.ready.set()

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            if not self.samples and self.error is None:
                self.error = (self.proc.stderr.read() or "sampler exited").strip().splitlines()[-1:]

    def summary(self, t0, t1):
        """Median SM clock and the union of active reasons over the samples taken
        between host times t0 and t1."""
        inside = [s for s in self.samples if t0 <= s[0] <= t1]
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0,
                    "source": "nvml", "error": self.error}
        mask = 0
        for s in inside:
            mask |= s[4]
        return {"sm_mhz": statistics.median(s[1] for s in inside), "sm_max_mhz": inside[-1][2],
                "power_w": statistics.median(s[3] for s in inside),
                "reasons": sorted(n for b, n in _REASON_BITS.items() if mask & b),
                "samples": len(inside), "gpus": len(self.keys), "source": "nvml",
                "window_s": round(t1 - t0, 4),
                "aggregate": "per sample: lowest SM clock, highest power, union of reasons over the GPUs"}


def make_params(n, seed, dev, rank=0, world=1, workload="config1"):
    """The Gaussians and cameras of one rank.

    config1: n Gaussians of config 1 per rank. With several ranks the shards sit
    side by side along x (12 units apart) and each rank's camera looks at its
    own shard, so every GPU renders one config-1 view of a scene that grows with
    the job (weak scaling); splats near the frustum edges still cross ranks
    through the exchange.
    config2 / config3: the whole scene of n Gaussians (4 / 8 cameras), each rank
    holding the strided shard [rank::world] of the Gaussians (the reference
    trainer's layout) and its consecutive share of the cameras: the job's work
    stays the same as ranks are added.
    config4: this rank's shard of n Gaussians and its cameras of the
    6M-Gaussian, 32-camera scene (the job's work stays the same)."""
    import torch

    from tests import _data

    if workload in ("config2", "config3"):
        d = _data.config2(N=n) if workload == "config2" else _data.config3(N=n)
        C = d["viewmats"].shape[0]
        assert C % world == 0, f"{workload}: {C} cameras do not split over {world} ranks"
        per = C // world
        for k in ("means", "quats", "scales", "opacities", "sh"):
            d[k] = d[k][rank::world].contiguous()
        d["viewmats"] = d["viewmats"][rank * per:(rank + 1) * per].contiguous()
        d["Ks"] = d["Ks"][rank * per:(rank + 1) * per].contiguous()
    elif workload == "config4":
        d = _data.config4(N=n, rank=rank, world=world)
    else:
        d = _data.config1(N=n, seed=seed)
    shift = 12.0 * (rank - (world - 1) / 2.0)
    if world > 1 and workload == "config1":
        d["means"][:, 0] += shift
        d["viewmats"] = d["viewmats"].clone()
        d["viewmats"][:, 0, 3] = -shift
    params = {
        "means": d["means"],
        "scales": torch.log(d["scales"]),
        "quats": d["quats"],
        "opacities": torch.logit(d["opacities"]),
        "sh": d["sh"],
    }
    params = {k: torch.nn.Parameter(v.to(dev).contiguous()) for k, v in params.items()}
    return params, d


def train_step(params, opt, viewmat, K, W, H, G, Ga, distributed=False, packed=True, mode=None):
    """One step through the public API: rasterization() forward, loss.backward()
    and (unless the workload's mode says otherwise) SelectiveAdam.step over the
    visible Gaussians (the reference trainer's visibility, simple_trainer.py)."""
    import torch

    import gsplat_b200

    mode = mode or STEP_MODES["config1"]
    render, alpha, meta = gsplat_b200.rasterization(
        params["means"], params["quats"], torch.exp(params["scales"]),
        torch.sigmoid(params["opacities"]), params["sh"], viewmat, K, W, H, near_plane=0.01,
        far_plane=100.0, sh_degree=3, packed=packed, distributed=distributed,
        render_mode=mode["render_mode"], rasterize_mode=mode["rasterize_mode"], absgrad=mode["absgrad"])
    loss = (render * G[..., :render.shape[-1]]).sum() + (alpha * Ga).sum()
    loss.backward()
    if not mode["adam"]:
        for p in params.values():
            p.grad = None
        return loss, meta
    n = params["means"].shape[0]
    if distributed:
        # the local shard's Gaussians that reached any rank's image: those with a
        # gradient (the packed ids after the exchange are the received splats')
        vis = params["means"].grad.ne(0).any(-1)
    elif packed:
        vis = torch.zeros(n, dtype=torch.bool, device=render.device)
        vis.index_fill_(0, meta["gaussian_ids"], True)
    else:
        vis = (meta["radii"] > 0).all(-1).any(0)
    opt.step(vis)
    opt.zero_grad(set_to_none=True)
    return loss, meta


def flop_per_pair(cdim):
    """Algorithmic FP32 work per contributing (pixel, splat) pair of the
    rasterizer: 20 + 2 CDIM forward, 50 + 6 CDIM backward (26 / 68 for RGB)."""
    return {"fwd": 20 + 2 * cdim, "bwd": 50 + 6 * cdim}


def cpu_scene(n, seed):
    """config-1 scene as float32 numpy arrays (same seeds as the GPU run)."""
    from tests import _data

    d = _data.config1(N=n, seed=seed)
    out = {k: (v.numpy() if hasattr(v, "numpy") else v) for k, v in d.items()}
    rng = __import__("numpy").random.default_rng(100 + seed)
    out["G"] = rng.standard_normal((1, d["height"], d["width"], 3)).astype("float32")
    out["Ga"] = rng.standard_normal((1, d["height"], d["width"], 1)).astype("float32")
    return out


def cpu_reference_step(sc, tile_row_stride=8):
    """One training step of the reference algorithm on the host cores (the CPU
    restatement in oracle/, OpenMP over all cores): projection, SH, AccuTile
    intersection + sort + offsets, rasterize forward/backward, the backward chain
    and the selective Adam update of every parameter. The rasterizer runs on every
    `tile_row_stride`-th row of tiles (a bounded, representative sample) and its
    time is scaled to the full image. Returns (seconds for a full step, detail)."""
    import numpy as np

    from oracle import oracle as O

    W, H = sc["width"], sc["height"]
    ts = 16
    tw, th = -(-W // ts), -(-H // ts)
    t = {}
    t0 = time.perf_counter()
    means, quats, scales, opac, sh = sc["means"], sc["quats"], sc["scales"], sc["opacities"], sc["sh"]
    vm, K = sc["viewmats"], sc["Ks"]
    radii, m2, dep, con, _ = O.projection_fwd(means, None, quats, scales, opac, vm, K, W, H,
                                              far_plane=100.0)
    valid = (radii > 0).all(-1)
    campos = -np.einsum("cji,cj->ci", vm[:, :3, :3], vm[:, :3, 3])
    dirs = means[None] - campos[:, None]
    coeffs = sh[None]
    raw = O.sh_fwd(3, dirs, coeffs, valid)
    colors = np.maximum(raw + 0.5, 0.0).astype(np.float32)
    op_eff = np.ascontiguousarray(opac[None])
    t["projection+sh"] = time.perf_counter() - t0
    t0 = time.perf_counter()
    _, keys, fids = O.isect_tiles(m2, radii, dep, ts, tw, th, conics=con, opacities=op_eff)
    offsets = O.isect_offset_encode(keys, 1, tw, th)
    t["isect+sort+offsets"] = time.perf_counter() - t0
    rows = np.arange(th) % tile_row_stride == 0
    masks = np.repeat(rows[:, None], tw, axis=1)[None]
    scale = masks.size / masks.sum()
    t0 = time.perf_counter()
    rc, ra, last = O.raster_fwd(m2, con, colors, op_eff, W, H, ts, offsets, fids, masks=masks)
    t["raster_fwd"] = (time.perf_counter() - t0) * scale
    t0 = time.perf_counter()
    v_m2, v_con, v_col, v_op, _ = O.raster_bwd(m2, con, colors, op_eff, W, H, ts, offsets, fids,
                                               ra, last, sc["G"], sc["Ga"], masks=masks)
    t["raster_bwd"] = (time.perf_counter() - t0) * scale
    t0 = time.perf_counter()
    v_col = v_col * (raw + 0.5 >= 0)
    v_coeffs, v_dirs = O.sh_bwd(3, dirs, coeffs, v_col, valid)
    v_means, _, v_quats, v_scales, _ = O.projection_bwd(
        means, None, quats, scales, vm, K, W, H, 0.3, radii, con, None, v_m2 * valid[..., None],
        np.zeros_like(dep), v_con * valid[..., None], None, viewmats_grad=False)
    v_means = v_means + v_dirs[0] * valid[0][:, None]
    t["backward chain"] = time.perf_counter() - t0
    t0 = time.perf_counter()
    vis = valid[0].astype(np.uint8)
    for p, g, lr in ((means, v_means, LRS["means"]), (quats, v_quats, LRS["quats"]),
                     (scales, v_scales, LRS["scales"]), (opac, v_op[0], LRS["opacities"]),
                     (sh, v_coeffs[0], LRS["sh"])):
        st = sc.setdefault("adam_state", {})
        m, v = st.setdefault(id(p), (np.zeros_like(p), np.zeros_like(p)))
        O.adam(p, g, m, v, vis, lr, 0.9, 0.999, 1e-15)
    t["adam"] = time.perf_counter() - t0
    return sum(t.values()), {k: round(v * 1e3, 2) for k, v in t.items()}


REF_BUDGET_S = 120.0  # wall time of the --impl reference steps (warm-up + timed)
CPU_BASELINE_STEPS = 3  # timed host steps of the cpu_baseline leg


def run_reference(args):
    """`--impl reference`: the reference algorithm timed on the host cores. Each
    step is a bounded sample of the config-1 step: the full scene through every
    stage, the rasterizer on every s-th row of tiles with its time scaled by the
    row fraction; one calibration step picks s (8, 16, 32 or 64) so that all
    warm-up and timed steps fit in REF_BUDGET_S where the host allows."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    if args.workload != "config1":
        print(json.dumps({"impl": "reference", "unavailable": "the host-core reference arm samples config1 only "
                          "(config3's ~238M intersections per step exceed a bounded host sample)"}), flush=True)
        return
    sc = cpu_scene(args.n, 1)
    W, H = sc["width"], sc["height"]
    _, cal = cpu_reference_step(sc, tile_row_stride=8)
    raster_full_s = (cal["raster_fwd"] + cal["raster_bwd"]) / 1e3  # scaled to the whole image
    other_s = sum(v for k, v in cal.items() if not k.startswith("raster")) / 1e3
    per_step = REF_BUDGET_S / max(1, args.warmup + args.steps)
    stride = 8
    while stride < 64 and other_s + raster_full_s / stride > per_step:
        stride *= 2
    for _ in range(args.warmup):
        cpu_reference_step(sc, tile_row_stride=stride)
    times, detail = [], None
    for _ in range(args.steps):
        dt, detail = cpu_reference_step(sc, tile_row_stride=stride)
        times.append(dt)
    ms = 1e3 * sum(times) / len(times)
    value = (W * H / 1e6) / (ms / 1e3)
    cores = os.cpu_count()
    sample = (f"config 1 ({args.n} Gaussians, 1297x840): projection, SH, isect, sort, backward chain and "
              f"Adam on the full scene; rasterizer forward/backward on every {stride}th tile row, scaled to "
              "the whole image")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "MPix/s",
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp32", "data": "synthetic (seeded config-1 distributions)",
        "config": {"workload": "config1: 1M Gaussians, 1297x840 pinhole fx=fy=1150, SH deg 3, "
                               "packed, fwd+bwd+SelectiveAdam",
                   "gaussians_per_rank": args.n, "cameras_per_rank": 1,
                   "parallelism": "host cores of rank 0", "stages_ms": detail},
        "cpu_baseline": {"value": value, "unit": "MPix/s", "cores": cores, "kind": "port",
                         "torch_threads": __import__("torch").get_num_threads(), "openmp_threads": cores,
                         "sample": sample},
        "e2e": {"value": value, "unit": "MPix/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def fp32_peak_tflops(dev):
    """Measured FP32 FMA throughput of this GPU (gsb_fp32_fma_probe)."""
    import torch

    from gsplat_b200.cuda import _backend

    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    blocks, threads, iters = sms * 8, 256, 4096
    out = torch.empty(blocks * threads, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    for _ in range(3):
        _backend.call("gsb_fp32_fma_probe", out.data_ptr(), blocks, threads, iters, stream)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    reps = 10
    for _ in range(reps):
        _backend.call("gsb_fp32_fma_probe", out.data_ptr(), blocks, threads, iters, stream)
    b.record()
    torch.cuda.synchronize(dev)
    sec = a.elapsed_time(b) / 1e3 / reps
    return blocks * threads * iters * 16 / sec / 1e12


def contributing_pairs(meta, W, H, dev):
    """Number of (pixel, splat) pairs that contribute to the image (alpha >= 1/255
    before each pixel's transmittance cut-off): the algorithmic work unit of both
    rasterizer kernels."""
    import torch

    from gsplat_b200.cuda import _backend

    offsets = meta["isect_offsets"].contiguous()
    fids = meta["flatten_ids"]
    ones = torch.zeros(meta["means2d"].shape[:-1] + (1,), device=dev)
    I = int(offsets.numel() // (offsets.shape[-1] * offsets.shape[-2]))
    th, tw = offsets.shape[-2:]
    renders = torch.empty((I, H, W, 1), device=dev)
    alphas = torch.empty((I, H, W, 1), device=dev)
    last = torch.empty((I, H, W), dtype=torch.int32, device=dev)
    counts = torch.empty((I, H, W), dtype=torch.int32, device=dev)
    _backend.call("gsb_rasterize_fwd_counted", I, 1, meta["means2d"].data_ptr(),
                  meta["conics"].data_ptr(), ones.data_ptr(), meta["opacities"].data_ptr(), None, None,
                  W, H, meta["tile_size"], tw, th, offsets.data_ptr(), fids.data_ptr(), fids.numel(),
                  renders.data_ptr(), alphas.data_ptr(), last.data_ptr(), counts.data_ptr(),
                  torch.cuda.current_stream(dev).cuda_stream)
    # pairs a per-pixel rasterizer evaluates in the backward: every entry of the
    # pixel's tile list up to its last contributor (none when nothing contributed)
    ts = meta["tile_size"]
    ys = torch.arange(H, device=dev) // ts
    xs = torch.arange(W, device=dev) // ts
    start = offsets.reshape(I, th, tw)[:, ys][:, :, xs].to(torch.int64)  # [I, H, W]
    walked = torch.where(counts > 0, last.to(torch.int64) - start + 1, torch.zeros_like(start))
    return int(counts.sum().item()), int(walked.sum().item())


def measured_hbm_gbs():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
            return float(json.load(fh)["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return None


def ncu_traffic(name):
    """DRAM bytes per launch recorded in profiles/<name>.md (line 'dram_bytes_per_launch: N')."""
    path = os.path.join(ROOT, "profiles", name + ".md")
    try:
        for line in open(path):
            if line.strip().startswith("dram_bytes_per_launch:"):
                return int(float(line.split(":", 1)[1]))
    except OSError:
        pass
    return None


SHARDED_STEPS = 10  # timed steps of the sharded config-4 measurement (at most --steps)


def measure_sharded(args, dev, rank, world, distributed):
    """The reference's sharded multi-GPU configuration at the
    job's N: 6M Gaussians split evenly over the ranks, 32 cameras at 1600x1200
    split over the ranks, rasterization(distributed=True) exchanging the
    projected splats, backward and SelectiveAdam on every rank. Total work is
    fixed, so the per-N values give the strong-scaling curve. W >= 3 warm-up
    steps, then min(K, SHARDED_STEPS) steps between barrier + synchronize, timed
    with CUDA events, max over ranks."""
    import torch
    import torch.distributed as dist

    import gsplat_b200

    n = 6_000_000 // world
    params, d = make_params(n, 1 + rank, dev, rank, world, "config4")
    W, H = d["width"], d["height"]
    viewmat, K = d["viewmats"].to(dev), d["Ks"].to(dev)
    n_cams = viewmat.shape[0]
    opt = gsplat_b200.SelectiveAdam([{"params": [p], "lr": LRS[k], "name": k} for k, p in params.items()],
                                    eps=1e-15, betas=(0.9, 0.999))
    g = torch.Generator(device=dev).manual_seed(200 + rank)
    G = torch.randn((n_cams, H, W, 3), device=dev, generator=g)
    Ga = torch.randn((n_cams, H, W, 1), device=dev, generator=g)
    bank = [(G, Ga), (-G, -Ga)]
    mode = STEP_MODES["config4"]

    def barrier():
        if distributed:
            dist.barrier()
        torch.cuda.synchronize()

    warm = max(3, min(args.warmup, 5))
    steps = max(1, min(args.steps, SHARDED_STEPS))
    for i in range(warm):
        train_step(params, opt, viewmat, K, W, H, *bank[i % 2], distributed, True, mode)
    barrier()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    mem0 = torch.cuda.memory_stats(dev)
    from gsplat_b200.cuda import _backend

    _backend.host_wait = [0.0, 0]
    wall0 = time.perf_counter()
    start.record()
    for i in range(steps):
        loss, meta = train_step(params, opt, viewmat, K, W, H, *bank[i % 2], distributed, True, mode)
    end.record()
    host_ms = (time.perf_counter() - wall0) * 1e3 / steps
    host_blocked_ms = _backend.host_wait[0] * 1e3 / steps
    _backend.host_wait = None
    barrier()
    mem1 = torch.cuda.memory_stats(dev)
    # device allocations (cudaMalloc) and allocator retries inside the timed steps
    alloc = {k: mem1.get(k, 0) - mem0.get(k, 0) for k in ("num_device_alloc", "num_device_free", "num_alloc_retries")}
    alloc["peak_gb"] = round(mem1.get("allocated_bytes.all.peak", 0) / 2**30, 1)
    ms = start.elapsed_time(end) / steps
    if distributed:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    mpix = world * n_cams * W * H / 1e6
    n_isects = torch.tensor([meta["isect_ids"].numel()], device=dev, dtype=torch.float64)
    if distributed:
        dist.all_reduce(n_isects)
    exchange = None
    if distributed:
        exchange = "peer memory" if os.environ.get("GSB_PEER_EXCHANGE", "1") != "0" else "nccl all_to_all"
    # per-entry-point device time of this rank, from two instrumented steps after
    # the timed ones (the exchange entry points include waiting for the others)
    _backend.timing = {}
    for i in range(2):
        train_step(params, opt, viewmat, K, W, H, *bank[i % 2], distributed, True, mode)
    barrier()
    ops = {name: round(sum(a.elapsed_time(b) for a, b in evs) / 2, 3) for name, evs in _backend.timing.items()}
    _backend.timing = None
    out = {"workload": WORKLOADS["config4"], "value": mpix / (ms / 1e3), "unit": "MPix/s",
           "ms_per_step": ms, "steps": steps, "warmup": warm, "scaling": "strong",
           "gaussians_per_rank": n, "cameras_per_rank": n_cams, "n_isects_job": int(n_isects.item()),
           "exchange": exchange, "timing": "CUDA events over the timed steps, max over ranks",
           "host_issue_ms_per_step": host_ms, "host_blocked_ms_per_step": host_blocked_ms,
           "allocator": alloc, "ops_ms_rank0": ops}
    del params, opt, bank, meta, loss
    torch.cuda.empty_cache()
    return out


def run_gsb(args):
    import torch
    import torch.distributed as dist

    import gsplat_b200
    from gsplat_b200.cuda import _backend

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    distributed = world > 1
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if distributed:
        import datetime

        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))

    params, d = make_params(args.n, 1 + rank, dev, rank, world, args.workload)
    packed = not args.dense
    mode = STEP_MODES[args.workload]
    W, H = d["width"], d["height"]
    viewmat = d["viewmats"].to(dev)
    K = d["Ks"].to(dev)
    n_cams = viewmat.shape[0]
    opt = gsplat_b200.SelectiveAdam([{"params": [p], "lr": LRS[k], "name": k} for k, p in params.items()],
                                    eps=1e-15, betas=(0.9, 0.999))
    # Upstream image gradients: N(0,1) images in antithetic pairs (G1, -G1, G2,
    # -G2) cycled step by step. Adam normalises its step by the gradient's RMS, so
    # any bank whose mean is not zero moves every parameter by about the learning
    # rate per step in a fixed direction (opacities and scales drift, splats grow
    # and the per-step work rises with the step count); with the pairs the
    # moments cancel and the scene, hence the work per step, stays that of
    # config 1 for any number of steps.
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    bank = []
    for _ in range(GRAD_BANK // 2):
        G_ = torch.randn((n_cams, H, W, 4 if mode["render_mode"] == "RGB+ED" else 3), device=dev, generator=g)
        Ga_ = torch.randn((n_cams, H, W, 1), device=dev, generator=g)
        bank += [(G_, Ga_), (-G_, -Ga_)]
    step_no = [0]

    def grads():
        G, Ga = bank[step_no[0] % GRAD_BANK]
        step_no[0] += 1
        return G, Ga

    def barrier():
        if distributed:
            dist.barrier()
        torch.cuda.synchronize()

    # rank 0 samples every rank's GPU in one child process
    keys = [gpu_key(dev)]
    if distributed:
        gathered = [None] * world
        dist.all_gather_object(gathered, keys[0])
        keys = gathered
    sampler = ClockSampler(keys if rank == 0 else [])
    sampler.__enter__()
    for _ in range(args.warmup):
        train_step(params, opt, viewmat, K, W, H, *grads(), distributed, packed, mode)
    barrier()

    # device-timed region: K full steps, inputs resident in HBM. Only the
    # rasterizer launches (the roofline's kernels) carry CUDA events here; every
    # entry-point call is counted. The per-entry-point breakdown comes from a
    # separate instrumented run below, since events around every call add host
    # time to a step whose issue is close to its device time.
    _backend.timing = {}
    _backend.timing_names = {"gsb_rasterize_fwd_ex", "gsb_rasterize_bwd_ex"}
    _backend.calls = {}
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    barrier()
    mem0 = torch.cuda.memory_stats(dev)
    _backend.host_wait = [0.0, 0]
    wall0 = time.perf_counter()
    clock0 = time.time()
    start.record()
    for _ in range(args.steps):
        loss, meta = train_step(params, opt, viewmat, K, W, H, *grads(), distributed, packed, mode)
    end.record()
    host_ms = (time.perf_counter() - wall0) * 1e3 / args.steps
    # host time blocked in the step's size reads (waiting for the device)
    host_blocked_ms = _backend.host_wait[0] * 1e3 / args.steps
    host_reads = _backend.host_wait[1] / args.steps
    _backend.host_wait = None
    barrier()
    mem1 = torch.cuda.memory_stats(dev)
    alloc = {k: mem1.get(k, 0) - mem0.get(k, 0) for k in ("num_device_alloc", "num_device_free", "num_alloc_retries")}
    clock1 = time.time()
    sampler.__exit__(None, None, None)
    ms = start.elapsed_time(end) / args.steps
    timing = _backend.timing
    calls = _backend.calls
    _backend.timing = None
    _backend.timing_names = None
    _backend.calls = None
    if distributed:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    mpix = world * n_cams * W * H / 1e6
    value = mpix / (ms / 1e3)
    # the rasterizer launches inside the timed region (CUDA events on their stream)
    raster_ms = {name: sum(s.elapsed_time(e) for s, e in evs) / args.steps for name, evs in timing.items()}

    # per-entry-point device time, from an instrumented run of the same step
    # after the timed region (events around every call)
    ops = {}
    n_ops_steps = min(args.steps, 20)
    _backend.timing = {}
    for _ in range(n_ops_steps):
        train_step(params, opt, viewmat, K, W, H, *grads(), distributed, packed, mode)
    barrier()
    for name, evs in _backend.timing.items():
        tot = sum(s.elapsed_time(e) for s, e in evs)
        ops[name] = {"ms_per_step": tot / n_ops_steps, "launch_calls": len(evs) // n_ops_steps}
    _backend.timing = None
    for name, v in raster_ms.items():
        ops[name]["ms_per_step_timed_region"] = v

    # end-to-end through the public API with host buffers: per step, the camera
    # and the upstream image gradients come from pinned host memory and the loss
    # is read back to the host. As in a training loop with a prefetching loader,
    # the inputs of step i + 1 are copied on a side stream while step i computes,
    # and the loss of step i is read once step i + 1 has been issued; every copy
    # and every read lies inside the timed region.
    e2e = None
    if not args.no_e2e:
        hv = viewmat.cpu().pin_memory()
        hK = K.cpu().pin_memory()
        hbank = [(G_.cpu().pin_memory(), Ga_.cpu().pin_memory()) for G_, Ga_ in bank]
        h2d = hv.numel() * 4 + hK.numel() * 4 + hbank[0][0].numel() * 4 + hbank[0][1].numel() * 4
        loss_host = [torch.empty((), dtype=torch.float32).pin_memory() for _ in range(2)]
        compute = torch.cuda.current_stream()
        copy_stream = torch.cuda.Stream()
        # two device copies of the inputs, used alternately; a copy into a slot
        # waits until the step that last read it has finished
        slots = [tuple(torch.empty_like(h, device=dev) for h in (hv, hK) + hbank[0]) for _ in range(2)]
        slot_free = [None, None]

        def prefetch(it):
            k = it % 2
            with torch.cuda.stream(copy_stream):
                if slot_free[k] is not None:
                    copy_stream.wait_event(slot_free[k])
                hG, hGa = hbank[it % GRAD_BANK]
                for dst, src in zip(slots[k], (hv, hK, hG, hGa)):
                    dst.copy_(src, non_blocking=True)
                ready = torch.cuda.Event()
                ready.record(copy_stream)
            return slots[k], ready

        barrier()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        copy_stream.wait_stream(compute)
        nxt = prefetch(0)
        pending = None
        losses = []
        for it in range(args.steps):
            (dv, dK, dG, dGa), ready = nxt
            compute.wait_event(ready)
            if it + 1 < args.steps:
                nxt = prefetch(it + 1)
            loss, _ = train_step(params, opt, dv, dK, W, H, dG, dGa, distributed, packed, mode)
            lh = loss_host[it % 2]
            lh.copy_(loss.detach(), non_blocking=True)
            done = torch.cuda.Event()
            done.record(compute)
            slot_free[it % 2] = done
            if pending is not None:
                pending[1].synchronize()
                losses.append(float(pending[0]))
            pending = (lh, done)
        pending[1].synchronize()
        losses.append(float(pending[0]))
        t1.record()
        barrier()
        ems = t0.elapsed_time(t1) / args.steps
        if distributed:
            t = torch.tensor([ems], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ems = float(t.item())
        assert len(losses) == args.steps and all(math.isfinite(x) for x in losses)
        e2e = {"value": mpix / (ems / 1e3), "unit": "MPix/s", "ms_per_step": ems,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4,
               "pipelining": "inputs of step i+1 copied on a side stream during step i; "
                             "loss of step i read after step i+1 is issued"}

    # the sharded configuration at this N (its own key; `value` stays the
    # headline workload's)
    sharded = None
    if args.workload == "config1" and not args.no_sharded:
        sharded = measure_sharded(args, dev, rank, world, distributed)

    roofline = None
    cpu_baseline = None
    if rank == 0 and ops.get("gsb_rasterize_bwd_ex"):
        pairs, walked = contributing_pairs(meta, W, H, dev)
        peak = fp32_peak_tflops(dev)
        t_bwd = raster_ms["gsb_rasterize_bwd_ex"] / 1e3
        cdim = 4 if mode["render_mode"] == "RGB+ED" else 3
        fpp = flop_per_pair(cdim)
        # the algorithmic unit of the survey's roofline table: every (pixel,
        # splat) pair a per-pixel rasterizer evaluates, i.e. the tile list up to
        # each pixel's last contributor (walked pairs)
        achieved = fpp["bwd"] * walked / t_bwd / 1e12
        achieved_contrib = fpp["bwd"] * pairs / t_bwd / 1e12
        traffic = ncu_traffic("raster_bwd_config1")
        roofline = {"kernel": f"raster_bwd_kernel<{cdim},4>", "bound": "fp32", "achieved": achieved,
                    "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                    "traffic": traffic,
                    "peak_source": "measured FP32 FMA probe (gsb_fp32_fma_probe) on this GPU; "
                                   "the kernel is FP32-issue bound (no tensor-core contraction, "
                                   "DRAM ~1%), so neither MEASURED_PEAKS figure applies",
                    "algorithmic": f"{fpp['bwd']} FLOP per evaluated (pixel, splat) pair; {walked} pairs per "
                                   "launch: each pixel's tile list up to its last contributor",
                    "contributing_pairs": pairs,
                    "achieved_contributing": achieved_contrib,
                    "frac_contributing": achieved_contrib / peak,
                    "contributing_note": "the stricter unit: only the pairs that pass the alpha test before "
                                         "each pixel's transmittance stop (this kernel culls most of the "
                                         "others before any arithmetic)",
                    "fwd": {"achieved": fpp["fwd"] * walked /
                            (raster_ms["gsb_rasterize_fwd_ex"] / 1e3) / 1e12,
                            "achieved_contributing": fpp["fwd"] * pairs /
                            (raster_ms["gsb_rasterize_fwd_ex"] / 1e3) / 1e12,
                            "unit": "TFLOP/s"}}
        hbm_peak = measured_hbm_gbs()
        if traffic and hbm_peak:
            gbs = traffic / t_bwd / 1e9
            roofline["hbm"] = {"achieved": gbs, "peak": hbm_peak, "unit": "GB/s", "frac": gbs / hbm_peak,
                               "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)"}
    if rank == 0 and world == 1 and not args.no_cpu and args.workload == "config1":
        sc = cpu_scene(args.n, 1)
        cpu_reference_step(sc)  # warm-up
        times = []
        for _ in range(CPU_BASELINE_STEPS):
            dt, detail = cpu_reference_step(sc)
            times.append(dt)
        dt = statistics.median(times)
        cpu_baseline = {"value": (W * H / 1e6) / dt, "unit": "MPix/s", "cores": os.cpu_count(),
                        "torch_threads": torch.get_num_threads(), "openmp_threads": os.cpu_count(),
                        "kind": "port", "ms_per_step": dt * 1e3, "steps": CPU_BASELINE_STEPS,
                        "step_ms_all": [round(t * 1e3, 1) for t in times], "stages_ms": detail,
                        "sample": f"config 1 step of the CPU restatement (oracle/), median of "
                                  f"{CPU_BASELINE_STEPS} steps after a warm-up: full projection, SH, "
                                  "isect, sort, backward chain, Adam; rasterizer on every 8th tile row "
                                  "scaled x8"}
    n_isects = int(meta["isect_ids"].numel()) if "isect_ids" in meta else None
    # visible (camera, Gaussian) pairs; distributed meta tensors keep their capacity rows
    nnz = (int(meta["gaussian_ids"].numel()) if meta.get("gaussian_ids") is not None and not distributed
           else None)
    # entry-point calls inside the timed region (each launches one or more kernels)
    launches = sum(calls.values()) // args.steps if calls else None

    result = {
        "metric": METRIC,
        "value": value,
        "unit": "MPix/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "weak" if args.workload == "config1" else "strong",
        "vs_baseline": None,
        "dtype": "fp32",
        "data": f"synthetic (seeded {args.workload} distributions, random-init Gaussians)",
        "config": {"workload": WORKLOADS[args.workload],
                   "gaussians_per_rank": int(params["means"].shape[0]), "cameras_per_rank": n_cams,
                   "parallelism": f"gaussian-sharded x{world}" if distributed else "single",
                   "packed": packed, "render_mode": mode["render_mode"],
                   "rasterize_mode": mode["rasterize_mode"], "absgrad": mode["absgrad"],
                   "optimizer": "SelectiveAdam" if mode["adam"] else None,
                   "l2": "inputs larger than L2 (params + Adam state ~700 MB)",
                   "visible_splats": nnz, "n_isects": n_isects},
        "clocks": sampler.summary(clock0, clock1),
        "e2e": e2e,
        "sharded": sharded,
        "roofline": roofline,
        "cpu_baseline": cpu_baseline,
        "gpu_launches": launches,
        "ops": ops,
        "ops_source": (f"CUDA events around every entry point over {n_ops_steps} further steps after the "
                       "timed region; ms_per_step_timed_region: the rasterizer inside it"),
        "host_issue_ms_per_step": host_ms,
        "host_blocked_ms_per_step": host_blocked_ms,
        "host_reads_per_step": host_reads,
        "allocator": alloc,
        "host_cpus": len(os.sched_getaffinity(0)),
    }
    if rank == 0:
        print(json.dumps(result), flush=True)
    if distributed:
        dist.barrier()
        dist.destroy_process_group()


def main():
    args = parse()
    if args.n is None:
        world = int(os.environ.get("WORLD_SIZE", "1"))
        args.n = {"config2": 500_000, "config3": 3_000_000, "config4": 6_000_000 // world}.get(args.workload,
                                                                                             1_000_000)
    if args.impl == "reference":
        run_reference(args)
        return
    run_gsb(args)


if __name__ == "__main__":
    main()
