"""Benchmark of the fused per-Gaussian backward-and-update step on B200.

Workload (one "step"): the fused per-Gaussian pass over 1,100,000 Gaussians,
SH degree 3 — SH colour VJP wrt coefficients and view direction, torch-fused
Adam on features_dc / features_rest, position adjoint into dm, and the
rotation / scaling / opacity activation VJPs with their Adam updates — with
the step counter advancing every step (bias corrections of steps 1, 2, ...),
moments carried over. Synthetic, seeded inputs with the distributions of the
fused-step configuration: features_dc ~ N(0.5, 0.1), features_rest ~
N(0, 0.05), means ~ U[-1, 1]^3 seen by one pinhole camera at (0, 0, -4)
(980x545, fov 60 deg: visibility and radii from the projection, clamped
channels from the SH colour), dL/dcolor ~ N(0, 1e-3), rotations ~ N(0, 1),
log-scales ~ U(-6, -2), opacity logits ~ N(-2, 1), activation seeds ~
N(0, 1e-4).

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
Multi-GPU runs go through torchrun; every rank steps its own 1.1M-Gaussian
shard (Gaussian-index sharding, no collective on the data path: weak scaling).
Prints one JSON line on rank 0.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import random
import statistics
import subprocess
import sys
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "clad-3dgs_b200"))

N_GAUSSIANS = 1_100_000
DEGREE = 3
BYTES_PER_GAUSSIAN = 1451          # SH 1207 + activations 244 (algorithmic)
H2D_BYTES_PER_GAUSSIAN = 767       # inputs of one host-buffer step
D2H_BYTES_PER_GAUSSIAN = 684       # outputs of one host-buffer step
METRIC = "Gaussians/s fused SH-grad+Adam & % HBM peak; train iters/s at 1/2/4/8 B200"
WORKLOAD = "fused per-Gaussian step (SH deg 3 VJP + Adam, activation VJPs + Adam)"
L2_NOTE = "inputs 1.60 GB per step exceed the 126 MB L2; no flush needed"
WIDTH, HEIGHT, FOV = 980, 545, math.radians(60.0)


def parse():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["native", "reference"], default="native")
    ap.add_argument("--workload", choices=["fused-step", "pixel-backward", "train-step"],
                    default="fused-step",
                    help="pixel-backward: the 1920x1080, 3M-Gaussian rasterizer pixel "
                         "backward configuration (timed for all accumulation modes)")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--e2e-chunk", type=int, default=131072,
                    help="Gaussians per host-buffer chunk (a multiple of 64)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--gaussians", type=int, default=N_GAUSSIANS,
                    help="Gaussians per GPU (smaller cases are for profiling only)")
    ap.add_argument("--no-train-step", action="store_true",
                    help="fused-step line without the attached training-step measurement")
    ap.add_argument("--train-gaussians", type=int, default=6_000_000,
                    help="train-step: replicated Gaussians (smaller cases are for profiling)")
    ap.add_argument("--view-offset", type=int, default=0,
                    help="train-step: rank r renders orbit camera (r + offset) mod 8")
    ap.add_argument("--exchange", choices=["peer", "collective"], default=None,
                    help="train-step: gradient exchange (default: peer memory on >1 GPU)")
    ap.add_argument("--sh-exchange", choices=["seeds", "colours", "grads"], default=None,
                    help="train-step: what a view publishes for the SH coefficients "
                         "(default: colours, the owners rendering each rank's next "
                         "colours, unless the exchange is collective)")
    ap.add_argument("--pixel-gaussians", type=int, default=3_000_000,
                    help="pixel-backward: 2D Gaussians (smaller cases are for profiling only)")
    ap.add_argument("--pixel-modes", default="2,1,0",
                    help="pixel-backward: accumulation modes to time, first is reported")
    return ap.parse_args()


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


# ---------------------------------------------------------------------------
# Clock sampling during the measurement.

class ClockSampler:
    """SM clock, power and throttle reasons of one GPU, sampled every 2 ms from
    a background thread through NVML (read-only queries) across warm-up and the
    timed loop; `timed()` marks the timed window, and the summary covers the
    samples inside it when there are at least three, else every sample under
    load. Falls back to nothing (reason "NVML unavailable") without NVML."""

    # NVML clocks-event-reason bits.
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, index: int, period_s: float = 0.002):
        self.index, self.period = index, period_s
        self.rows, self.window = [], [None, None]
        self.handle = self.thread = None
        self.stop = False

    def _open(self):
        import pynvml
        import torch

        pynvml.nvmlInit()
        props = torch.cuda.get_device_properties(self.index)
        bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
        try:
            handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except pynvml.NVMLError:
            handle = pynvml.nvmlDeviceGetHandleByIndex(self.index)
        self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM)
        return pynvml, handle

    def _run(self, nvml, handle):
        while not self.stop:
            try:
                self.rows.append((time.monotonic(),
                                  nvml.nvmlDeviceGetClockInfo(handle, nvml.NVML_CLOCK_SM),
                                  nvml.nvmlDeviceGetPowerUsage(handle) / 1000.0,
                                  nvml.nvmlDeviceGetCurrentClocksEventReasons(handle)))
            except nvml.NVMLError:
                pass
            time.sleep(self.period)

    def __enter__(self):
        import threading

        try:
            nvml, self.handle = self._open()
        except Exception:  # no NVML on this machine
            self.handle = None
            return self
        self.thread = threading.Thread(target=self._run, args=(nvml, self.handle), daemon=True)
        self.thread.start()
        return self

    def __exit__(self, *exc):
        self.stop = True
        if self.thread is not None:
            self.thread.join(timeout=5)

    def timed(self, begin: bool):
        """Marks the start (True) or end (False) of the timed region."""
        self.window[0 if begin else 1] = time.monotonic()

    def summary(self):
        if self.handle is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["NVML unavailable"]}
        lo, hi = self.window
        inside = [r for r in self.rows if lo is not None and hi is not None and lo <= r[0] <= hi]
        window = "timed region"
        if len(inside) < 3:
            inside = [r for r in self.rows if r[2] > 200] or list(self.rows)
            window = "warm-up and timed region"
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["no samples"]}
        reasons = sorted({name for r in inside for bit, name in self.REASONS.items()
                          if r[3] & bit})
        return {"sm_mhz": statistics.median(r[1] for r in inside), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(inside), "window": window,
                "power_w_median": statistics.median(r[2] for r in inside), "source": "NVML"}


# ---------------------------------------------------------------------------
# Synthetic state of one shard.

def make_state(n, device, seed):
    import torch

    g = torch.Generator(device=device).manual_seed(seed)
    randn = lambda *s: torch.randn(s, generator=g, device=device)
    rand = lambda *s: torch.rand(s, generator=g, device=device)
    means = rand(n, 3) * 2 - 1
    camera = torch.tensor([0.0, 0.0, -4.0], device=device)
    dc = randn(n, 1, 3) * 0.1 + 0.5
    rest = randn(n, 15, 3) * 0.05
    log_scale = rand(n, 3) * 4 - 6
    rotation = randn(n, 4)
    opacity = randn(n, 1) - 2
    # Pinhole camera at (0,0,-4) looking down +z: visibility and pixel radii.
    rel = means - camera
    focal = (WIDTH / 2) / math.tan(FOV / 2)
    depth = rel[:, 2]
    px = rel[:, 0] / depth * focal
    py = rel[:, 1] / depth * focal
    inside = (depth > 0.2) & (px.abs() < WIDTH / 2 + 64) & (py.abs() < HEIGHT / 2 + 64)
    sigma_px = 3.0 * log_scale.exp().max(1).values * focal / depth
    radii = torch.where(inside, torch.ceil(sigma_px).clamp_min(1), 0).to(torch.int32)
    # Clamped channels: SH colour + 0.5 < 0 (the renderer's convention).
    dirs = rel / rel.norm(dim=1, keepdim=True)
    from_sh = _eval_sh3(torch.cat((dc, rest), 1).transpose(1, 2), dirs) + 0.5
    clamped = (from_sh < 0).contiguous()
    state = dict(
        means=means.contiguous(), radii=radii.contiguous(), clamped=clamped,
        camera=camera, seed=(randn(n, 3) * 1e-3).contiguous(),
        dm=torch.zeros(n, 3, device=device), dc=dc.contiguous(), rest=rest.contiguous(),
        dc_first=torch.zeros(n, 1, 3, device=device), dc_second=torch.zeros(n, 1, 3, device=device),
        rest_first=torch.zeros(n, 15, 3, device=device),
        rest_second=torch.zeros(n, 15, 3, device=device))
    params = [rotation.contiguous(), log_scale.contiguous(), opacity.contiguous()]
    state["act"] = dict(
        params=params,
        seeds=[(randn(*p.shape) * 1e-4).contiguous() for p in params],
        saved=[rotation.norm(2, dim=1, keepdim=True).contiguous(), log_scale.exp().contiguous(),
               opacity.sigmoid().contiguous()],
        first=[torch.zeros_like(p) for p in params],
        second=[torch.zeros_like(p) for p in params],
        rates=[0.001, 0.005, 0.025])
    return state


def _eval_sh3(sh, dirs):
    """Degree-3 real-SH colour of sh [n, 3, 16] along unit dirs [n, 3]; used
    only to draw the clamped flags of the synthetic inputs."""
    x, y, z = dirs[:, 0:1], dirs[:, 1:2], dirs[:, 2:3]
    xx, yy, zz = x * x, y * y, z * z
    basis = [0.28209479177387814 + 0 * x, -0.4886025119029199 * y, 0.4886025119029199 * z,
             -0.4886025119029199 * x, 1.0925484305920792 * x * y,
             -1.0925484305920792 * y * z, 0.31539156525252005 * (2 * zz - xx - yy),
             -1.0925484305920792 * x * z, 0.5462742152960396 * (xx - yy),
             -0.5900435899266435 * y * (3 * xx - yy), 2.890611442640554 * x * y * z,
             -0.4570457994644658 * y * (4 * zz - xx - yy),
             0.3731763325901154 * z * (2 * zz - 3 * xx - 3 * yy),
             -0.4570457994644658 * x * (4 * zz - xx - yy),
             1.445305721320277 * z * (xx - yy), -0.5900435899266435 * x * (xx - 3 * yy)]
    out = 0
    for j, b in enumerate(basis):
        out = out + b * sh[..., j]
    return out


def step_bias(t):
    import numpy as np

    return float(np.float32(1 - 0.9 ** t)), float(np.float32(math.sqrt(1 - 0.999 ** t)))


def run_step(consume, s, t):
    b1, b2 = step_bias(t)
    a = s["act"]
    consume.gaussian_step(s["means"], s["radii"], s["clamped"], s["camera"], s["seed"],
                          s["dm"], s["dc"], s["rest"], s["dc_first"], s["dc_second"],
                          s["rest_first"], s["rest_second"], bias1=b1, bias2_sqrt=b2,
                          degree=DEGREE, act_parameters=a["params"], act_seeds=a["seeds"],
                          act_saved=a["saved"], act_first=a["first"], act_second=a["second"],
                          act_rates=a["rates"], act_bias1=[b1] * 3, act_bias2=[b2] * 3)


def fused_config(gaussians_per_gpu, world):
    """The `config` of the fused-step line (the same in both arms)."""
    return {"workload": WORKLOAD, "gaussians_per_gpu": gaussians_per_gpu, "sh_degree": DEGREE,
            "camera": "980x545 pinhole, fov 60",
            "parallelism": f"Gaussian-index shards x{world}", "l2": L2_NOTE}


def measured_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def ncu_traffic():
    """(DRAM bytes of one 1.1M-Gaussian launch of the fused kernel, note) from
    the committed ncu capture."""
    path = ROOT / "profiles" / "fused_gaussian_step_traffic.json"
    if not path.exists():
        return None, None
    try:
        data = json.loads(path.read_text())
        return float(data["bytes_per_launch_at_1.1M"]), data.get("note")
    except (ValueError, KeyError):
        return None, None


def cpu_baseline(budget_s=15.0):
    sys.path.insert(0, str(ROOT / "oracle"))
    import torch_cpu_path

    probe = torch_cpu_path.time_cpu_path(20_000, steps=2, warmup=1)
    per_g = probe["total_s"] / (probe["n"] * probe["steps"])
    n = int(min(N_GAUSSIANS, max(20_000, budget_s / 12 / per_g)))
    res = torch_cpu_path.time_cpu_path(n, steps=10, warmup=1)
    return {"value": res["gaussians_per_s"], "unit": "Gaussians/s", "cores": res["threads"],
            "kind": "port",
            "sample": f"{n} Gaussians (of {N_GAUSSIANS}), 10 timed steps after 1 warm-up; "
                      "torch CPU eval_sh + autograd + torch.optim.Adam, fp32"}


# ---------------------------------------------------------------------------

def native_arm(args):
    import torch
    import torch.distributed as dist

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=device)
    import consume
    import _native as native

    n_g = args.gaussians
    state = make_state(n_g, device, seed=42 + rank)
    torch.cuda.synchronize()
    t = 0
    with ClockSampler(local) as clocks:
        for _ in range(args.warmup):
            t += 1
            run_step(consume, state, t)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        stream = torch.cuda.current_stream()
        events = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
        clocks.timed(True)
        events[0].record(stream)
        for k in range(args.steps):
            t += 1
            run_step(consume, state, t)
            events[k + 1].record(stream)
        torch.cuda.synchronize()
        clocks.timed(False)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
    clock_summary = clocks.summary()
    per_step = [events[k].elapsed_time(events[k + 1]) for k in range(args.steps)]
    elapsed_ms = events[0].elapsed_time(events[-1])
    fault = native.fault_status()
    local_ms = torch.tensor([elapsed_ms], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(local_ms, op=dist.ReduceOp.MAX)
    elapsed_ms = float(local_ms.item())

    e2e = e2e_measurement(args, device, consume) if rank == 0 and not args.no_e2e else None
    del state
    train = None
    if not args.no_train_step:
        torch.cuda.empty_cache()
        train = measure_train_step(args, steps=24, warmup=8, with_e2e=False)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    total_g = n_g * world * args.steps
    # One persistent launch per step, plus the one-tile kernel when the
    # Gaussian count is not a multiple of the tile size.
    tile = native.describe()["tile_gaussians"]
    launches_per_step = 1 + (1 if n_g % tile else 0)
    value = total_g / (elapsed_ms / 1e3)
    peak, peak_kind = measured_peaks()
    mean_step_s = statistics.mean(per_step) / 1e3
    achieved = BYTES_PER_GAUSSIAN * n_g / mean_step_s / 1e9
    traffic, traffic_note = ncu_traffic()
    line = {
        "metric": METRIC, "value": value, "unit": "Gaussians/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": elapsed_ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32+f64",
        "data": "synthetic (seeded; distributions of the fused-step configuration)",
        "config": fused_config(n_g, world),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic,
                     "traffic_note": traffic_note,
                     "peak_kind": f"{peak_kind} hbm_gbs (copy, burst)",
                     "algorithmic_bytes_per_gaussian": BYTES_PER_GAUSSIAN,
                     "kernel_time_ms": mean_step_s * 1e3},
        "clocks": clock_summary,
        "e2e": e2e,
        "gpu_launches": launches_per_step * args.steps,
        "device_fault_word": fault,
    }
    if train is not None:
        line["train_step"] = {k: train[k] for k in ("metric", "value", "unit", "ms_per_step",
                                                    "iters_per_s", "steps", "warmup",
                                                    "exchange", "loss", "per_rank",
                                                    "gpu_launches")}
        line["train_step"]["config"] = train["config"]
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline()
    print(json.dumps(line), flush=True)


def e2e_measurement(args, device, consume):
    """Same metric through the C ABI with pinned host buffers: every step copies
    its inputs in and its results out (chunked, overlapped) inside the timing."""
    import torch

    s = make_state(N_GAUSSIANS, device, seed=1042)
    host = {k: (v.cpu().pin_memory() if torch.is_tensor(v) else v) for k, v in s.items()
            if k != "act"}
    act = {k: ([x.cpu().pin_memory() for x in v] if k != "rates" else v)
           for k, v in s["act"].items()}
    del s
    chunk = args.e2e_chunk
    ws = torch.empty(consume.host_step_workspace(chunk), dtype=torch.uint8, device=device)

    def one(t):
        b1, b2 = step_bias(t)
        consume.gaussian_step_host(
            host["means"], host["radii"], host["clamped"], host["camera"], host["seed"],
            host["dm"], host["dc"], host["rest"], host["dc_first"], host["dc_second"],
            host["rest_first"], host["rest_second"], bias1=b1, bias2_sqrt=b2, degree=DEGREE,
            act_parameters=act["params"], act_seeds=act["seeds"], act_saved=act["saved"],
            act_first=act["first"], act_second=act["second"], act_rates=act["rates"],
            act_bias1=[b1] * 3, act_bias2=[b2] * 3, workspace=ws, chunk=chunk)

    steps = max(3, args.e2e_steps)
    for t in range(1, 3):
        one(t)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for t in range(3, 3 + steps):
        one(t)
    end.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    h2d = H2D_BYTES_PER_GAUSSIAN * N_GAUSSIANS + 12
    d2h = D2H_BYTES_PER_GAUSSIAN * N_GAUSSIANS
    ceiling = pcie_ceiling(device)
    # Both directions run concurrently, so the step cannot be shorter than the
    # slower direction at the measured concurrent copy rates.
    floor_ms = max(h2d / ceiling["both_h2d_gbs"], d2h / ceiling["both_d2h_gbs"]) / 1e6
    return {"value": N_GAUSSIANS * steps / (ms / 1e3), "unit": "Gaussians/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "steps": steps, "ms_per_step": ms / steps,
            "pcie": dict(ceiling, copy_floor_ms=floor_ms, frac_of_copy_floor=floor_ms / (ms / steps)),
            "path": f"clad3dgs_gaussian_step_host (C ABI), pinned host buffers, {chunk:,}-"
                    "Gaussian chunks on 3 streams"}


def pcie_ceiling(device, nbytes=512 << 20, reps=5):
    """Pinned host<->device copy rates (GB/s): each direction alone and both at
    once on two streams (cudaMemcpyAsync through torch), best of `reps`."""
    import torch

    host_in = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    host_out = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    dev_in = torch.empty(nbytes, dtype=torch.uint8, device=device)
    dev_out = torch.empty(nbytes, dtype=torch.uint8, device=device)
    s1, s2 = torch.cuda.Stream(device), torch.cuda.Stream(device)

    def timed(fn):
        best = float("inf")
        for _ in range(reps):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            fn()
            torch.cuda.synchronize()
            best = min(best, time.perf_counter() - t0)
        return best

    def both():
        with torch.cuda.stream(s1):
            dev_in.copy_(host_in, non_blocking=True)
        with torch.cuda.stream(s2):
            host_out.copy_(dev_out, non_blocking=True)

    t_h2d = timed(lambda: dev_in.copy_(host_in, non_blocking=True))
    t_d2h = timed(lambda: host_out.copy_(dev_out, non_blocking=True))
    t_both = timed(both)
    return {"h2d_gbs": nbytes / t_h2d / 1e9, "d2h_gbs": nbytes / t_d2h / 1e9,
            "both_h2d_gbs": nbytes / t_both / 1e9, "both_d2h_gbs": nbytes / t_both / 1e9,
            "bytes_per_copy": nbytes}


def reference_arm(args):
    """The reference's CPU path (eval_sh + autograd + torch.optim.Adam) on host
    cores; rank 0 only."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    sys.path.insert(0, str(ROOT / "oracle"))
    import torch_cpu_path

    probe = torch_cpu_path.time_cpu_path(20_000, steps=2, warmup=1)
    per_g = probe["total_s"] / (probe["n"] * probe["steps"])
    budget = 150.0 / max(1, args.steps + args.warmup)
    n = int(min(N_GAUSSIANS, max(1024, budget / per_g)))
    res = torch_cpu_path.time_cpu_path(n, steps=args.steps, warmup=args.warmup)
    sample = (f"{n} Gaussians per step (of {N_GAUSSIANS}), {args.steps} timed steps after "
              f"{args.warmup} warm-up, on the host cores of rank 0; torch CPU eval_sh + "
              "autograd + torch.optim.Adam")
    line = {
        "impl": "reference", "metric": METRIC, "value": res["gaussians_per_s"],
        "unit": "Gaussians/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": res["total_s"] * 1e3 / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded; distributions of the fused-step configuration)",
        "config": fused_config(N_GAUSSIANS, world),
        "cpu_baseline": {"value": res["gaussians_per_s"], "unit": "Gaussians/s",
                         "cores": res["threads"], "kind": "port", "sample": sample},
        "e2e": {"value": res["gaussians_per_s"], "unit": "Gaussians/s",
                "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def make_2d_scene(n, width, height, device, seed):
    """Depth-sorted 2D Gaussians of the pixel-backward configuration: means
    uniform over the image, per-axis standard deviations lognormal(1.5, 0.7) px
    at a uniform angle, opacities U(0.05, 0.99), colours U(0, 1)."""
    import torch

    g = torch.Generator(device=device).manual_seed(seed)
    rand = lambda *s: torch.rand(s, generator=g, device=device)
    randn = lambda *s: torch.randn(s, generator=g, device=device)
    mean2d = rand(n, 2) * torch.tensor([width, height], device=device, dtype=torch.float32)
    s1 = torch.exp(1.5 + 0.7 * randn(n))
    s2 = torch.exp(1.5 + 0.7 * randn(n))
    th = rand(n) * math.pi
    c, s = torch.cos(th), torch.sin(th)
    a = c * c * s1 * s1 + s * s * s2 * s2
    b = c * s * (s1 * s1 - s2 * s2)
    d = s * s * s1 * s1 + c * c * s2 * s2
    det = a * d - b * b
    conic_opacity = torch.stack([d / det, -b / det, a / det, 0.05 + 0.94 * rand(n)], 1)
    radii = torch.ceil(3 * torch.maximum(s1, s2)).to(torch.int32)
    return dict(mean2d=mean2d.contiguous(), conic_opacity=conic_opacity.contiguous(),
                rgb=rand(n, 3).contiguous(), depth=(1 + 99 * rand(n)).contiguous(),
                radii=radii.contiguous())


def pixel_backward_arm(args):
    import torch

    import rasterizer
    import _native as native

    device = torch.device("cuda", 0)
    W, H, n = 1920, 1080, args.pixel_gaussians
    scene = make_2d_scene(n, W, H, device, seed=4)
    bg = torch.zeros(3, device=device)
    num, color, _inv, state = rasterizer.forward_2d(
        scene["mean2d"], scene["conic_opacity"], scene["rgb"], scene["depth"], scene["radii"],
        W, H, bg)
    gen = torch.Generator(device=device).manual_seed(5)
    dpix = (torch.randn((3, H, W), generator=gen, device=device) * 1e-3).contiguous()
    grads = dict(dmean2d=torch.zeros(n, 3, device=device), dconic=torch.zeros(n, 4, device=device),
                 dopacity=torch.zeros(n, device=device), dcolor=torch.zeros(n, 3, device=device))
    tiles = ((W + 15) // 16) * ((H + 15) // 16)
    # Algorithmic bytes of one pass: per pixel dL/dpix 12 + final T 4 + last
    # contributor 4; per tile instance its index 4 + features 36 (xy 8,
    # conic/opacity 16, rgb 12; inverse depth unused without an inverse-depth
    # adjoint); per Gaussian the nine adjoints written 36; tile ranges 8.
    algorithmic = H * W * 20 + num * 40 + n * 36 + tiles * 8
    peak, peak_kind = measured_peaks()
    results = {}
    modes = [int(m) for m in args.pixel_modes.split(",")]
    for mode in modes:
        for _ in range(args.warmup):
            rasterizer.render_backward_2d(state, dpix, grads, mode)
        torch.cuda.synchronize()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        ev[0].record()
        for _ in range(args.steps):
            rasterizer.render_backward_2d(state, dpix, grads, mode)
        ev[1].record()
        torch.cuda.synchronize()
        ms = ev[0].elapsed_time(ev[1]) / args.steps
        results[mode] = ms
    ms = results[modes[0]]
    names = {2: "converged_warp_reduction", 1: "full_warp_only (reference helper)",
             0: "per_lane_atomics"}
    # Atomics of one pass (a counting pass replays the walk's contribution
    # test; it is not timed). Nine adjoint fields without an inverse-depth
    # adjoint: colour 3, screen mean 2, conic 3, opacity 1.
    fields = 9
    counts = rasterizer.count_accumulation_2d(state)
    per_mode = {0: counts["pairs"] * fields, 1: counts["mode1_per_field"] * fields,
                2: counts["mode2_reductions"] * fields}
    atomics = {
        "contributing_pairs": counts["pairs"],
        "reference_sites_times_pairs": 8 * counts["pairs"],
        "per_lane_atomics_mode0": per_mode[0],
        "full_warp_only_atomics_mode1": per_mode[1],
        "converged_reduction_instructions_mode2": counts["mode2_reductions"],
        "converged_reduction_atomics_mode2": per_mode[2],
        "atomics_per_pass": per_mode[modes[0]],
        "atomics_per_s": per_mode[modes[0]] / (ms / 1e3),
        "atomic_instructions_per_s": (counts["mode2_reductions"] if modes[0] == 2
                                      else per_mode[modes[0]]) / (ms / 1e3),
        "note": "lane-level atomic operations per pass; mode 2 issues one multi-lane "
                "atomic instruction per (warp, Gaussian) covering all nine fields",
    }
    line = {
        "metric": "rasterizer pixel backward, Gaussians/s (1920x1080, one pass over every "
                  "2D Gaussian)",
        "value": n / (ms / 1e3), "unit": "Gaussians/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "data": "synthetic (seeded 2D Gaussians of the pixel-backward configuration)",
        "config": {"workload": f"pixel backward, 1920x1080, 16x16 tiles, {n:,} depth-sorted "
                               "2D Gaussians, radii lognormal(1.5, 0.7) px, opacity U(0.05,0.99), "
                               "T stop 1e-4, dL/dpixel N(0,1e-3)",
                   "tile_instances": num, "accumulation_mode": modes[0],
                   "ms_per_mode": {names[m]: results[m] for m in modes}},
        "atomics": atomics,
        "roofline": {"bound": "hbm", "limiter": "instruction issue and latency (the ncu "
                                                "summary of this kernel: DRAM < 1% of peak)",
                     "achieved": algorithmic / (ms / 1e3) / 1e9,
                     "peak": peak, "unit": "GB/s",
                     "frac": algorithmic / (ms / 1e3) / 1e9 / peak,
                     "algorithmic_bytes": algorithmic, "peak_kind": peak_kind},
        "device_fault_word": native.fault_status(),
    }
    print(json.dumps(line), flush=True)


def train_values(n, device, seed=3):
    """Gaussians of the 8-view data-parallel configuration: means U[-1,1]^3,
    f_dc N(0.5, 0.1), f_rest N(0, 0.05), log-scales U(-6, -2), quaternions
    N(0, 1), opacity logits N(-2, 1)."""
    import torch

    g = torch.Generator(device=device).manual_seed(seed)
    sh = torch.randn(n, 16, 3, generator=g, device=device) * 0.05
    sh[:, 0] = 0.5 + 0.1 * torch.randn(n, 3, generator=g, device=device)
    return dict(xyz=torch.rand(n, 3, generator=g, device=device) * 2 - 1,
                sh=sh.reshape(n, 48),
                scaling=torch.rand(n, 3, generator=g, device=device) * 4 - 6,
                rotation=torch.randn(n, 4, generator=g, device=device),
                opacity=torch.randn(n, 1, generator=g, device=device) - 2)


TRAIN_GAUSSIANS, TRAIN_W, TRAIN_H = 6_000_000, 1920, 1080
# Kernels of ours per training step: activate, preprocess, SH colour, depth keys,
# row gather, row emission, row layout, tile counts, tile totals, tile ranges,
# instance placement, render forward, L1 loss, render backward, preprocess
# backward, then with SH gradients: SH backward, shard update; with colour
# seeds: seeds, SH + position update, shard update of the other groups; the
# colour form has no SH colour pass (CUB's scans, sorts and reductions and
# NCCL's barriers are library launches).
TRAIN_LAUNCHES_PER_STEP = {"grads": 17, "seeds": 18, "colours": 17}


def train_step_arm(args):
    """Full data-parallel training step: one 1920x1080 view per GPU of 6M
    replicated Gaussians (SH degree 3), L1 loss, rasterizer backward, exchange +
    sharded Adam. Value: views trained per second over all GPUs."""
    import torch
    import torch.distributed as dist

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    line = measure_train_step(args, args.steps, args.warmup, not args.no_e2e)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def measure_train_step(args, steps, warmup, with_e2e):
    """Times the data-parallel training step on every rank (process group, if
    any, already up); returns the JSON line on rank 0, None elsewhere."""
    import torch
    import torch.distributed as dist

    rank, world, local = dist_env()
    device = torch.device("cuda", local)
    import _native as native
    from data_parallel import DataParallelTrainer, ShardedAdam, orbit_camera

    n = args.train_gaussians
    values = train_values(n, device)
    # Colour form unless the exchange is the collective one over several ranks.
    form = args.sh_exchange
    if form is None:
        form = "grads" if args.exchange == "collective" and world > 1 else "colours"
    trainer = DataParallelTrainer(values, exchange=args.exchange, device=device,
                                  sh_exchange=form)
    del values
    # The 8 orbit cameras and a fixed random target per camera. Like a trainer
    # drawing its views from a shuffled stack, step k uses a seeded permutation
    # of the 8 cameras (the same on every rank) and rank r renders its r-th
    # camera: every step's views are distinct and every GPU count sees the same
    # random mix of axis and diagonal views (the diagonal views cost more).
    cams = [orbit_camera(v, 8, width=TRAIN_W, height=TRAIN_H, device=device) for v in range(8)]
    targets = []
    for v in range(8):
        gen = torch.Generator(device=device).manual_seed(100 + v)
        targets.append(torch.rand(3, TRAIN_H, TRAIN_W, generator=gen, device=device))
    counter = [0]
    coloured = trainer.adam.sh_exchange == "colours"

    def draw():
        order = random.Random(1000 + counter[0]).sample(range(8), 8)
        v = (order[rank % 8] + args.view_offset) % 8
        counter[0] += 1
        return v

    # The colour form declares each step's next view: the views are drawn one
    # step ahead, in the same sequence.
    ahead = [draw() if coloured else None]

    def view():
        if not coloured:
            return draw(), None
        v, ahead[0] = ahead[0], draw()
        return v, ahead[0]

    def step_once(target=None):
        v, nxt = view()
        tgt = targets[v] if target is None else target(v)
        if coloured:
            return trainer.step(cams[v], tgt, next_camera=cams[nxt])
        return trainer.step(cams[v], tgt)

    stream = torch.cuda.current_stream()

    per_rank = {}

    def max_over_ranks(x, name=None):
        t = torch.tensor([x], device=device, dtype=torch.float64)
        if world > 1:
            every = torch.empty(world, device=device, dtype=torch.float64)
            dist.all_gather_into_tensor(every, t)
            values = every.tolist()
        else:
            values = [x]
        if name:
            per_rank[name] = [round(v, 4) for v in values]
        return max(values)

    def bracket():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    first_loss = None
    instances = 0
    with ClockSampler(local) as clocks:
        for k in range(warmup):
            loss, instances = step_once()
            if k == 0:
                first_loss = float(loss.item())
        bracket()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        clocks.timed(True)
        ev[0].record(stream)
        for _ in range(steps):
            loss, instances = step_once()
        ev[1].record(stream)
        torch.cuda.synchronize()
        clocks.timed(False)
        bracket()
    step_ms = max_over_ranks(ev[0].elapsed_time(ev[1]) / steps, "step_ms")
    last_loss = float(loss.item())
    # The exchange + update alone (gradients of a real backward in place).
    exchange_steps = max(3, min(steps, 20))
    total = backward_total = 0.0
    # The update kernels alone (between the exchange's two barriers).
    update_events = []
    plain_update = trainer.adam._update

    def timed_update(step):
        u0, u1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        u0.record(stream)
        plain_update(step)
        u1.record(stream)
        update_events.append((u0, u1))

    trainer.adam._update = timed_update
    for _ in range(exchange_steps):
        b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        b0.record(stream)
        v, nxt = view()
        trainer.backward(cams[v], targets[v])
        b1.record(stream)
        bracket()
        backward_total += b0.elapsed_time(b1)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if coloured:
            trainer.adam.next_camera.copy_(cams[nxt].campos)
            trainer._declared = cams[nxt]
        e0.record(stream)
        trainer.adam.step()
        e1.record(stream)
        torch.cuda.synchronize()
        total += e0.elapsed_time(e1)
    trainer.adam._update = plain_update
    exchange_ms = max_over_ranks(total / exchange_steps, "exchange_ms")
    update_ms = max_over_ranks(sum(u0.elapsed_time(u1) for u0, u1 in update_events)
                               / max(len(update_events), 1), "update_kernels_ms")
    max_over_ranks(backward_total / exchange_steps, "render_and_backward_ms")
    adam = trainer.adam
    baseline_ms = None
    if world > 1 and adam.exchange == "peer":
        # NCCL baseline of the same exchange: reduce-scatter, update, all-gather.
        other = ShardedAdam(n, exchange="collective", device=device)
        other.activate()
        bracket()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for _ in range(2):
            other.step()
        bracket()
        e0.record(stream)
        for _ in range(exchange_steps):
            other.step()
        e1.record(stream)
        bracket()
        baseline_ms = max_over_ranks(e0.elapsed_time(e1) / exchange_steps)
        other.close()
        del other
    # End to end: each step's target comes from pinned host memory and the
    # loss goes back to the host.
    e2e = None
    if with_e2e:
        host_targets = [t.cpu().pin_memory() for t in targets]
        dev_target = torch.empty_like(targets[0])
        loss_host = torch.empty(1, pin_memory=True)

        def staged(v):
            dev_target.copy_(host_targets[v], non_blocking=True)
            return dev_target

        e2e_steps = max(3, min(steps, 20))
        bracket()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(e2e_steps):
            loss, _ = step_once(staged)
            loss_host.copy_(loss, non_blocking=True)
        e1.record(stream)
        bracket()
        e2e_ms = max_over_ranks(e0.elapsed_time(e1) / e2e_steps)
        e2e = {"value": world / (e2e_ms / 1e3), "unit": "views/s",
               "h2d_bytes_per_step": host_targets[0].numel() * 4, "d2h_bytes_per_step": 4,
               "ms_per_step": e2e_ms}
    inst = torch.tensor([float(instances)], device=device, dtype=torch.float64)
    if world > 1:
        every = torch.empty(world, device=device, dtype=torch.float64)
        dist.all_gather_into_tensor(every, inst)
        instances_all = [int(v) for v in every.tolist()]
    else:
        instances_all = [int(instances)]
    fault = native.fault_status()
    padded, share = adam.padded, adam.share
    trainer.close()
    if rank != 0:
        return None
    # Exchange roofline, per GPU, in units of one Gaussian of its share (R
    # ranks). Across NVLink per direction, per peer: out, the share's updated
    # parameters (236 B; colour form: 44 B without the SH, and 12 B of
    # colours); in, the peer's view inputs (236 B of gradients; seed and colour
    # forms: 16 B colour seeds and 44 B of geometry gradients). From this GPU's
    # HBM: its moments read and written (944 B), its replica's parameters of
    # the share read and written (2 x 236 B), its view inputs read by all R
    # owners, the peers' parameter stores into its replica, and in colour form
    # its colours (12 B) and the share's clamp bits (8 B). The bound is the
    # slower of the two against the measured peer copy (770 GB/s per
    # direction) and the measured HBM copy.
    floats = 59
    seeded = adam.sh_exchange != "grads"
    coloured = adam.sh_exchange == "colours"
    inputs = (16 + 11 * 4) if seeded else floats * 4  # per Gaussian and view
    outputs = (11 * 4 + 12) if coloured else floats * 4
    link = (world - 1) * share * max(inputs, outputs)
    hbm = share * (944 + 2 * floats * 4 + world * inputs + (world - 1) * outputs
                   + (20 if coloured else 0))
    peak, peak_kind = measured_peaks()
    link_s, hbm_s = link / 770e9, hbm / (peak * 1e9)
    if link_s > hbm_s:
        exchange_roof = {"bound": "nvlink", "achieved": link / (exchange_ms / 1e3) / 1e9,
                         "peak": 770.0, "unit": "GB/s",
                         "peak_kind": "measured peer copy per direction"}
    else:
        exchange_roof = {"bound": "hbm", "achieved": hbm / (exchange_ms / 1e3) / 1e9,
                         "peak": peak, "unit": "GB/s", "peak_kind": peak_kind}
    exchange_roof.update(frac=max(link_s, hbm_s) / (exchange_ms / 1e3),
                         link_bytes_per_direction=link, hbm_bytes=hbm,
                         bound_ms=max(link_s, hbm_s) * 1e3)
    line = {
        "metric": "data-parallel training step, views/s (one 1920x1080 view per GPU)",
        "value": world / (step_ms / 1e3), "unit": "views/s", "n_gpus": world,
        "steps": steps, "warmup": warmup, "ms_per_step": step_ms,
        "iters_per_s": 1e3 / step_ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32+f64",
        "data": "synthetic (seeded; 6M Gaussians of the 8-view configuration, random targets)",
        "config": {"workload": f"{n:,} Gaussians SH degree 3 replicated, one {TRAIN_W}x{TRAIN_H} "
                               "view per GPU per step from 8 cameras on a radius-4 orbit (fov "
                               "60; step k: a seeded permutation of the cameras, rank r takes "
                               "its r-th), L1 loss, rasterizer backward, exchange + sharded "
                               "torch-fused Adam",
                   "exchange": adam.exchange, "sh_exchange": adam.sh_exchange,
                   "padded_gaussians": padded,
                   "share_per_gpu": share, "tile_instances_rank0": instances,
                   "l2": "parameters 1.4 GB per replica exceed the 126 MB L2"},
        "loss": {"first": first_loss, "last": last_loss},
        "per_rank": dict(per_rank, tile_instances=instances_all),
        "exchange": {"ms": exchange_ms, "update_kernels_ms": update_ms,
                     "nccl_baseline_ms": baseline_ms,
                     "roofline": exchange_roof},
        "clocks": clocks.summary(),
        "e2e": e2e,
        "gpu_launches": TRAIN_LAUNCHES_PER_STEP[adam.sh_exchange] * steps,
        "device_fault_word": fault,
    }
    return line


def main():
    args = parse()
    if args.impl == "reference":
        reference_arm(args)
    elif args.workload == "pixel-backward":
        pixel_backward_arm(args)
    elif args.workload == "train-step":
        train_step_arm(args)
    else:
        native_arm(args)


if __name__ == "__main__":
    main()
