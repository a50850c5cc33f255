#!/usr/bin/env python
"""Benchmark of the B200-native splatting path: fwd+bwd views/s at 500k Gaussians (SH
degree 3), 1024 x 768 — the training step of instantsplat-rs's `Trainer` (one view: forward,
SSIM/L1 loss, backward, Adam + scale clamp) on the benchmark's config 2.

    python bench.py [--gpus N --steps K --warmup W]          # this library (default)
    python bench.py --impl reference [--steps K --warmup W]  # the CPU restatement, host cores

One JSON line on rank 0. `value` is device-timed throughput with every input resident in
HBM; `e2e` is the same step through the public API as the reference's caller runs it
(camera from the host, pose refinement on: the 56-byte camera gradient and the loss read
back every step). At N > 1 each rank trains its own views (weak scaling); by default one
kernel per rank sums its share of every rank's gradients over NVLink peer memory, steps Adam
on it and stores the parameters into every rank's buffer (splat_b200/sharding.py, "peer").
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time
from datetime import timedelta
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path[:0] = [str(ROOT / "splatting-rs_b200"), str(ROOT / "oracle")]

METRIC = "fwd+bwd views/sec @500k Gaussians 1024x768 (1/2/4/8 GPU); fwd Mpix/s @3M"
UNIT = "views/s"
CONFIG_INDEX = 2
MEASURED_PEAKS = ROOT / "MEASURED_PEAKS.json"
FALLBACK_HBM_GBS = 6650.0
SMS = 148
FP32_LANES_PER_SM = 128
# FP32 instructions per (pixel, Gaussian) pair the blend kernels evaluate, counted from
# their inner loops (rasterize_forward.wgsl:58-77, rasterize_backward.wgsl:166-200): an
# FMA counts as one. The backward adds a 9-float warp reduction per (Gaussian, warp).
FORWARD_OPS_PER_PAIR = 20
BACKWARD_OPS_PER_PAIR = 48

# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per launch of the heaviest kernels,
# from one ncu --set full capture of this workload each (profiles/blend_kernels_config2.txt,
# profiles/project_config2.txt, profiles/project_backward_adam_config2.txt; cold caches, so an
# upper bound on the in-bench traffic).
NCU_TRAFFIC_BYTES = {"blend_backward": 78.9e6, "blend_forward": 28.8e6, "backward_adam": 836.7e6,
                     "project": 138.1e6, "emit": 42.1e6}


def parse_args():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=None,
                   help="timed steps (default 1000; 20 for --impl reference, whose steps take ~1 s each)")
    p.add_argument("--warmup", type=int, default=None, help="untimed steps first (default 10; 3 for the reference)")
    p.add_argument("--impl", choices=["b200", "reference"], default="b200")
    p.add_argument("--scale", type=float, default=1.0, help="Gaussian count scale (1.0 = the benchmark)")
    p.add_argument("--views", type=int, default=None, help="use only the first V views (small profiling cases)")
    p.add_argument("--e2e-steps", type=int, default=300)
    p.add_argument("--cpu-seconds", type=float, default=20.0, help="CPU-baseline sample budget")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-forward-3m", action="store_true", help="skip the forward-only config-3 measurement")
    p.add_argument("--forward-batches", type=int, default=3, help="timed passes over config 3's 64 cameras")
    p.add_argument("--no-densify", action="store_true", help="skip the device densification timing")
    p.add_argument("--no-web-example", action="store_true", help="skip the timing on the reference's example scene")
    p.add_argument("--no-config5", action="store_true", help="skip the 6M-Gaussian multi-GPU configuration")
    p.add_argument("--config5-iterations", type=int, default=2, help="timed iterations of config 5 (128 views each)")
    p.add_argument("--exchange", choices=["auto", "peer", "sharded", "allreduce"], default="auto",
                   help="multi-GPU exchange (auto: peer where the Gaussians split evenly, else all-reduce)")
    p.add_argument("--tiles", choices=["ellipse", "rectangle"], default="ellipse",
                   help="tile culling: the ellipse's tiles only (the same images and gradients, shorter lists) "
                        "or the reference's whole bounding rectangles")
    args = p.parse_args()
    if args.steps is None:
        args.steps = 20 if args.impl == "reference" else 1000
    if args.warmup is None:
        args.warmup = 3 if args.impl == "reference" else 10
    return args


def peaks() -> dict:
    if MEASURED_PEAKS.exists():
        data = json.loads(MEASURED_PEAKS.read_text())
        return {"hbm_gbs": float(data["hbm_gbs"]), "source": "measured", "sm_max_mhz": float(data.get("sm_max_mhz", 1965))}
    return {"hbm_gbs": FALLBACK_HBM_GBS, "source": "fallback", "sm_max_mhz": 1965.0}


# ------------------------------------------------------------------------------ clocks


class ClockSampler:
    """SM clock, power and clock-event reasons sampled during the timed region: through NVML
    every 2 ms in a thread (so that short regions get samples too), or, where NVML is not
    available, nvidia-smi every 100 ms. Entered before the ranks' barrier and the start event,
    left after the stop event has completed."""

    QUERY = (
        "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
        "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
        "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
    )
    # NVML clock-event reason bits (nvml.h: nvmlClocksEventReason*).
    REASON_BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
                   "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80}

    def __init__(self, device: int):
        self.device = device
        self.samples: list[tuple[float, float, float, int]] = []  # sm MHz, max MHz, W, reasons
        self.source = None
        self._stop = None
        self._thread = None
        self._proc = None
        self._file = None

    def _nvml_handle(self):
        import pynvml
        import torch

        pynvml.nvmlInit()
        try:
            uuid = str(torch.cuda.get_device_properties(self.device).uuid)
            return pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
        except Exception:  # noqa: BLE001 — fall back to the index among the visible devices
            visible = os.environ.get("CUDA_VISIBLE_DEVICES")
            index = int(visible.split(",")[self.device]) if visible else self.device
            return pynvml.nvmlDeviceGetHandleByIndex(index)

    def __enter__(self):
        import threading

        try:
            import pynvml

            handle = self._nvml_handle()
            self._stop = threading.Event()

            def run() -> None:
                while not self._stop.is_set():
                    try:
                        sm = pynvml.nvmlDeviceGetClockInfo(handle, pynvml.NVML_CLOCK_SM)
                        top = pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM)
                        watts = pynvml.nvmlDeviceGetPowerUsage(handle) / 1000.0
                        reasons = pynvml.nvmlDeviceGetCurrentClocksEventReasons(handle)
                        self.samples.append((float(sm), float(top), watts, int(reasons)))
                    except Exception:  # noqa: BLE001
                        pass
                    self._stop.wait(0.002)

            self._thread = threading.Thread(target=run, daemon=True)
            self._thread.start()
            self.source = "nvml, 2 ms"
        except Exception:  # noqa: BLE001 — no NVML: nvidia-smi
            self._file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            try:
                self._proc = subprocess.Popen(
                    ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                     "-lms", "100"], stdout=self._file, stderr=subprocess.DEVNULL)
                self.source = "nvidia-smi, 100 ms"
            except OSError:
                self._proc = None
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=5)
        if self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()
        if self._file is not None:
            self._file.flush()
            self._file.seek(0)
            for line in self._file.read().splitlines():
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    bits = 0
                    for name, flag in zip(["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown",
                                           "sw_power_cap"], parts[5:9]):
                        if flag.lower().startswith("active"):
                            bits |= self.REASON_BITS[name]
                    self.samples.append((float(parts[1]), float(parts[2]), float(parts[3]), bits))
                except ValueError:
                    continue
            os.unlink(self._file.name)
        return False

    def summary(self) -> dict:
        sm = [x[0] for x in self.samples]
        reasons = sorted({name for *_, bits in self.samples for name, bit in self.REASON_BITS.items() if bits & bit})
        return {
            "sm_mhz": float(np.median(sm)) if sm else None,
            "sm_max_mhz": max((x[1] for x in self.samples), default=None),
            "power_w_max": max((x[2] for x in self.samples), default=None),
            "samples": len(sm),
            "reasons": reasons,
            "source": self.source,
        }


def host_cores() -> dict:
    """The host threads this process may run on (all of them are given to the CPU legs,
    whatever OMP_NUM_THREADS says) and the CPU model."""
    model = None
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return {"threads": len(os.sched_getaffinity(0)), "model": model}


def libraries_loaded() -> list[str]:
    """The shared libraries of this repository mapped into the process."""
    try:
        maps = Path("/proc/self/maps").read_text()
    except OSError:
        return []
    found = {line.split()[-1] for line in maps.splitlines() if line.endswith(".so") and str(ROOT) in line}
    return sorted(str(Path(p).relative_to(ROOT)) for p in found)


def peer_copy_gbs(src_device: int, dst_device: int, mib: int = 512, reps: int = 10) -> float:
    """One-direction NVLink bandwidth between two GPUs of this node: a plain device-to-device
    copy (cudaMemcpyAsync through torch's copy_) of `mib` MiB from `src_device` to
    `dst_device`, `reps` times, timed with CUDA events on the source device's stream after
    three untimed copies. GB/s (10^9 bytes per second)."""
    import torch

    src = torch.ones(mib << 18, dtype=torch.float32, device=f"cuda:{src_device}")
    dst = torch.empty(mib << 18, dtype=torch.float32, device=f"cuda:{dst_device}")
    with torch.cuda.device(src_device):
        for _ in range(3):
            dst.copy_(src)
        torch.cuda.synchronize(src_device)
        torch.cuda.synchronize(dst_device)
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(reps):
            dst.copy_(src)
        stop.record()
        torch.cuda.synchronize(src_device)
        torch.cuda.synchronize(dst_device)
        ms = start.elapsed_time(stop)
    bytes_moved = reps * src.numel() * 4
    del src, dst
    torch.cuda.empty_cache()
    return bytes_moved / (ms / 1000.0) / 1e9


# --------------------------------------------------------------------------- workload


def build_ground_truth(ctx, scene, options_fn):
    """Targets: the scene's ground-truth cloud rendered by this library, masked at
    coverage 0.5 (pose_tests.rs:168-189), as loss::ground_truth_rgba lays them out."""
    import torch

    import splat_b200 as sb

    cams = scene.cameras
    w, h = cams[0].width, cams[0].height
    truth = torch.from_numpy(scene.truth.to_packed()).cuda()
    rast = sb.Rasterizer(ctx, truth, len(scene.truth), w, h, None, 0, options_fn())
    gt = np.empty((len(cams), h * w, 4), np.float32)
    for v, cam in enumerate(cams):
        rgbt = rast.render(cam).rgbt.reshape(-1, 4)
        mask = ((1.0 - rgbt[:, 3]) > 0.5).astype(np.float32)
        gt[v, :, :3] = rgbt[:, :3] * mask[:, None]
        gt[v, :, 3] = mask
    rast.close()
    del truth
    return gt


def cpu_baseline(scene, gt: np.ndarray, seconds: float = 0.0, steps: int | None = None, warmup: int = 0) -> dict:
    """The CPU oracle's training step (or_train_step: the reference's kernels restated in C++,
    OpenMP on every host thread this process may use) on the same workload, views in order.
    With `steps`: `warmup` untimed steps, then exactly `steps` timed ones; otherwise steps
    until the sample budget `seconds` is spent (at least 2). Camera records and learning rates
    come from the oracle and numpy, not from this library."""
    import oracle

    from splat_b200.camera import cameras_extent
    from splat_b200.gaussians import param_stride
    from splat_b200.optimizer import LEARNING_RATES_3DGS

    cores = host_cores()
    oracle.set_threads(cores["threads"])
    cams = scene.cameras
    records = [oracle.camera_of(c) for c in cams]
    params = scene.cloud.to_packed().copy()
    m = np.zeros_like(params)
    v = np.zeros_like(params)
    deg = scene.cloud.sh_degree
    stride = param_stride(deg)
    extent = np.float32(cameras_extent(cams))
    max_log = float(np.log(np.float32(0.02) * extent))
    aniso = float(np.log(np.float32(10.0)))
    lr = oracle.learning_rates_by_slot(LEARNING_RATES_3DGS.to_c(), extent, stride)
    done = 0

    def one_step() -> float:
        nonlocal done
        view = done % len(cams)
        t0 = time.perf_counter()
        oracle.train_step(params, deg, records[view], gt[view].reshape(-1), m, v, lr, done + 1, max_log, aniso)
        done += 1
        return time.perf_counter() - t0

    for _ in range(warmup):
        one_step()
    times = []
    start = time.perf_counter()
    if steps is not None:
        times = [one_step() for _ in range(steps)]
    else:
        while len(times) < 2 or (time.perf_counter() - start < seconds and len(times) < 64):
            times.append(one_step())
    total = sum(times)
    first = warmup
    return {
        "steps": len(times),
        "value": len(times) / total,
        "unit": UNIT,
        "cores": cores["threads"],
        "cpu": cores["model"],
        "kind": "port",
        "sample": f"{len(times)} full training steps of the benchmark workload (views {first} to "
                  f"{first + len(times) - 1} mod {len(cams)}, after {warmup} untimed) by the C++ oracle, "
                  f"OpenMP on {cores['threads']} host threads, {total:.1f} s",
        "ms_per_step": 1000.0 * total / len(times),
    }


def cpu_densify(params: np.ndarray, first: np.ndarray, second: np.ndarray, stats: np.ndarray, stride: int,
                extent: float, max_count: int, settings) -> dict:
    """The reference's densification flow on the host (training.rs:238-266): the CPU
    restatement of densify (single-threaded, as the Rust), on buffers already read back."""
    import oracle

    t0 = time.perf_counter()
    _, _, _, report = oracle.densify(params, first, second, stats, stride, extent, max_count, settings.to_c(), 0, 0)
    return {"ms": 1000.0 * (time.perf_counter() - t0), "cores": 1, "kind": "port", "after": report["after"]}


def densify_timing(ctx, rast, adam, extent: float, gaussians: int) -> dict:
    """One densification of the trained state on the device (sp_densify_plan + apply with
    DENSIFY_SHORT_RUN, the outputs allocated), timed on the host around the call (it
    synchronises) and per kernel with CUDA events; the state itself is left unchanged."""
    import torch

    import splat_b200 as sb

    settings = sb.DENSIFY_SHORT_RUN
    max_count = settings.max_count(gaussians)
    walls = []
    for _ in range(4):
        torch.cuda.synchronize()
        ctx.profile(True)
        t0 = time.perf_counter()
        out = sb.densify(rast, adam, float(extent), max_count, settings, False, 0)
        walls.append(1000.0 * (time.perf_counter() - t0))
        ctx.profile(False)
        kernel_ms, launches = ctx.read_profile()["densify"]
        del out
    report = sb.densify(rast, adam, float(extent), max_count, settings, False, 0).report
    return {"wall_ms": float(np.median(walls[1:])), "kernel_ms": kernel_ms, "launches": launches,
            "before": report.before, "after": report.after, "cloned": report.cloned, "split": report.split,
            "pruned": report.pruned_transparent + report.pruned_oversized,
            "what": "sp_densify_plan + sp_densify_apply (classify, select, scan, write; the report read back) "
                    "of the benchmark's trained state with DENSIFY_SHORT_RUN; median of 3 after one warm-up"}


def run_reference(args) -> None:
    """--impl reference: the reference's CPU arithmetic (the oracle port: the reference itself
    is Rust + WGSL on wgpu and has no CPU path that runs here) on every host thread, exactly
    --warmup untimed and --steps timed training steps. Rank 0 alone runs; this library's
    shared object is never loaded (targets rendered and cameras formed by the oracle)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle

    from splat_b200 import scenes

    scene = scenes.config(CONFIG_INDEX, scale=args.scale)
    cams = scene.cameras
    truth = scene.truth.to_packed()
    deg = scene.truth.sh_degree
    oracle.set_threads(host_cores()["threads"])
    needed = min(len(cams), args.warmup + args.steps)
    gt = np.zeros((len(cams), cams[0].width * cams[0].height, 4), np.float32)
    for view in range(needed):
        rgbt = oracle.render(truth, deg, oracle.camera_of(cams[view]))["image"].reshape(-1, 4)
        mask = ((1.0 - rgbt[:, 3]) > 0.5).astype(np.float32)
        gt[view, :, :3] = rgbt[:, :3] * mask[:, None]
        gt[view, :, 3] = mask
    result = cpu_baseline(scene, gt, steps=args.steps, warmup=args.warmup)
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": result["value"],
        "unit": UNIT,
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")),
        "steps": result["steps"],
        "warmup": args.warmup,
        "ms_per_step": result["ms_per_step"],
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": config_dict(scene, 1),
        "cpu_baseline": {k: result[k] for k in ("value", "unit", "cores", "cpu", "kind", "sample")},
        "e2e": {"value": result["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "libraries_loaded": libraries_loaded(),
    }
    print(json.dumps(line), flush=True)


EXCHANGES = {
    "peer": "gradients of each rank's share summed over NVLink peer memory, Adam on the share and the "
            "parameters stored into every rank's buffer, in one kernel per rank",
    "sharded": "gradients reduce-scattered, Adam sharded by Gaussians, parameters all-gathered (NCCL)",
    "allreduce": "gradients all-reduced (NCCL), the Adam step on every rank",
}


def config_dict(scene, world: int, exchange: str = "peer") -> dict:
    cam = scene.cameras[0]
    return {
        "workload": f"config 2: {len(scene.cloud)} Gaussians SH{scene.cloud.sh_degree}, {cam.width}x{cam.height}, "
                    f"{len(scene.cameras)} views; one step = forward + SSIM/L1 loss + backward + Adam per view",
        "gaussians": len(scene.cloud),
        "sh_degree": scene.cloud.sh_degree,
        "width": cam.width,
        "height": cam.height,
        "views": len(scene.cameras),
        "views_per_step": world,
        "parallelism": (f"view-sharded dp{world}: {EXCHANGES[exchange]}" if world > 1 else "single GPU"),
        "l2": "working set (params, gradients, Adam moments: >0.4 GB) larger than the 126 MB L2",
    }


# ----------------------------------------------------------------- config 5 (multi-GPU)


CONFIG5 = dict(gaussians=6_000_000, width=1600, height=1200, views=128, seed=4)


def config5_throughput(args, ctx, comm, rank: int, world: int, max_over_ranks, barrier) -> dict:
    """BASELINE's multi-GPU configuration: 6M Gaussians SH degree 3, 128 views of 1600 x 1200
    on a sphere; each iteration every rank accumulates the gradients of its 128 / world views
    (a contiguous block, in view order), then one exchange and one Adam step (sp_exchange_step
    through the library's communicator; the whole Adam step on one GPU). Total work per
    iteration is fixed whatever the GPU count (strong scaling). The scene is drawn on the GPU
    (scenes.packed_clustered_device, seed 4); the targets are this library's renders of its
    perturbed copy, masked at coverage 0.5, each rank holding its own views' targets only.
    Device-timed (CUDA events, max over ranks) over `config5_iterations` iterations after one."""
    import torch

    import splat_b200 as sb
    from splat_b200 import scenes
    from splat_b200.sharding import ViewShardedStep

    c = CONFIG5
    n, w, h, views = c["gaussians"], c["width"], c["height"], c["views"]
    if views % world:
        return {"skipped": f"{views} views do not split over {world} GPUs"}
    block = views // world
    device = torch.device("cuda", ctx.device)
    params, truth = scenes.packed_clustered_device(n, c["seed"], device, perturb=True)
    cams = scenes.sphere_cameras(views, 4.0, w, h)
    uniforms = [cam.uniform() for cam in cams]
    mine = list(range(rank * block, (rank + 1) * block))
    culling = sb.SP_TILES_ELLIPSE if args.tiles == "ellipse" else sb.SP_TILES_RECTANGLE
    gt = torch.empty((block, w * h, 4), dtype=torch.float32, device=device)
    painter = sb.Rasterizer(ctx, truth, n, w, h, None, 0,
                            sb.default_options(sh_degree=3, backward_mode=sb.SP_BWD_ATOMIC, tile_culling=culling))
    for k, v in enumerate(mine):
        rgbt = torch.from_numpy(painter.render(uniforms[v]).rgbt.reshape(-1, 4)).to(device)
        mask = ((1.0 - rgbt[:, 3]) > 0.5).float()
        gt[k, :, :3] = rgbt[:, :3] * mask[:, None]
        gt[k, :, 3] = mask
    painter.close()
    del truth
    opts = sb.default_options(sh_degree=3, backward_mode=sb.SP_BWD_ATOMIC, tile_culling=culling,
                              accumulate_gradients=True)
    rast = sb.Rasterizer(ctx, params, n, w, h, gt.reshape(-1), block, opts)
    extent = float(sb.cameras_extent(cams))
    adam = sb.Adam(ctx, params, rast, n, sb.LEARNING_RATES_3DGS, extent, sh_degree=3)
    step = ViewShardedStep(rast, adam, params, uniforms, rank, world, comm=comm, views_per_rank=block,
                           loss_index=lambda v: v - rank * block)
    iterations = 200
    step(0, sb.position_rate_factor(0, iterations))
    ctx.profile(True)
    step(1, sb.position_rate_factor(1, iterations))
    ctx.profile(False)
    profile = {k: v for k, v in ctx.read_profile().items() if v[1]}
    meta = rast.read_intersections_unchecked()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(ctx.device) as clocks:
        barrier()
        start.record()
        for i in range(args.config5_iterations):
            step(2 + i, sb.position_rate_factor(2 + i, iterations))
        stop.record()
        torch.cuda.synchronize()
    ms = max_over_ranks(start.elapsed_time(stop))
    exchange_mode = getattr(step.exchange, "mode", "adam")
    out = {
        "value": views * args.config5_iterations / (ms / 1000.0),
        "unit": "views/s",
        "workload": f"config 5: {n} Gaussians SH3, {views} views {w}x{h} on a sphere; one iteration = every "
                    f"view's forward, loss and backward accumulated ({block} per GPU), one exchange and one Adam step",
        "scaling": "strong: 128 views per iteration whatever the GPU count",
        "n_gpus": world,
        "iterations": args.config5_iterations,
        "ms_per_iteration": ms / args.config5_iterations,
        "exchange": exchange_mode if world > 1 else "none (one GPU: the Adam step)",
        "intersections_last_view": int(meta.count),
        "overflow": bool(meta.overflow),
        "kernels_ms_per_iteration": {k: v[0] for k, v in profile.items()},
        "clocks": clocks.summary(),
        "data": "synthetic: drawn on the GPU with torch's generator (seed 4), configs 3-4's distributions",
    }
    step.exchange.close() if world > 1 else None
    rast.close()
    adam.close()
    del params, gt
    torch.cuda.empty_cache()
    return out


# ------------------------------------------------------------------- the example scene


WEB_EXAMPLE = ROOT / "tests" / "golden" / "web_example"
# The reference's published step time on this scene (instantsplat-rs/src/gpu.rs:22-25):
# examples/step_timing.rs, native wgpu on Metal, shader bounds checks off, Apple M5.
WEB_EXAMPLE_PUBLISHED_MS = 36.0


def web_example_timing(ctx, steps: int = 300, warmup: int = 10) -> dict | None:
    """instantsplat-rs/examples/step_timing.rs on its own scene (web/example: the splat.ply of a
    fit run, 222,909 SH-degree-0 Gaussians, 6 views of 392 x 518 with their PNG targets):
    LEARNING_RATES_SHORT_RUN, views cycled in order, the position rate decayed over `steps`,
    after `warmup` steps; "fixed" poses (one sp_train_step per step, nothing read back until
    the end) and "refined" poses (sp_train_step_host_poses: the camera gradient read back and
    the host pose step every step). Both with the benchmark's options, timed with CUDA events
    around the loop and a final read of the loss, as the example times its loop."""
    import torch

    import splat_b200 as sb
    from splat_b200 import io as splat_io

    if not all((WEB_EXAMPLE / name).is_file() for name in ("splat.ply", "cameras.json", "input_view5.png")):
        return None
    cloud, cameras, gt_host = splat_io.read_fit_run(WEB_EXAMPLE)
    w, h = cameras[0].width, cameras[0].height
    gt = torch.from_numpy(gt_host.reshape(-1)).cuda()
    packed = torch.from_numpy(cloud.to_packed()).cuda()
    rates = sb.LEARNING_RATES_SHORT_RUN
    extent = float(sb.cameras_extent(cameras))
    uniforms = [c.uniform() for c in cameras]
    out = {}
    for label in ("fixed", "refined"):
        params = packed.clone()
        opts = sb.default_options(sh_degree=0, backward_mode=sb.SP_BWD_ATOMIC, tile_culling=sb.SP_TILES_ELLIPSE)
        rast = sb.Rasterizer(ctx, params, len(cloud), w, h, gt, len(cameras), opts)
        adam = sb.Adam(ctx, params, rast, len(cloud), rates, extent)
        poses = sb.PoseRefinement(cameras, rates, extent) if label == "refined" else None

        def step(i: int, total: int) -> None:
            view = i % len(cameras)
            factor = sb.position_rate_factor(i, total)
            if poses is None:
                rast.train_step(adam, uniforms[view], view, factor, read_back=False)
            else:
                rast.train_step_host_poses(adam, poses, view, factor)

        for i in range(warmup):
            step(i % len(cameras), steps)
        rast.read_loss()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for i in range(steps):
            step(i, steps)
        loss = rast.read_loss()
        stop.record()
        torch.cuda.synchronize()
        ms = start.elapsed_time(stop) / steps
        out[label] = {"ms_per_step": ms, "views_per_s": 1000.0 / ms, "loss_after": loss.total}
        rast.close()
        del adam, params
    return {
        "scene": f"instantsplat-rs/web/example: {len(cloud)} Gaussians SH0, {len(cameras)} views {w}x{h}, "
                 "LEARNING_RATES_SHORT_RUN",
        "steps": steps,
        "warmup": warmup,
        **out,
        "published_reference_ms_per_step": WEB_EXAMPLE_PUBLISHED_MS,
        "published_reference": "36 ms/step, Apple M5, wgpu/Metal, shader bounds checks off "
                               "(instantsplat-rs/src/gpu.rs:22-25; examples/step_timing.rs)",
        "speedup_vs_published_fixed": WEB_EXAMPLE_PUBLISHED_MS / out["fixed"]["ms_per_step"],
    }


# ------------------------------------------------------------------------------- main


def forward_throughput(args, ctx, rank: int, world: int, max_over_ranks, barrier) -> dict:
    """BASELINE's "fwd Mpix/s @3M": config 3 (3M Gaussians, SH degree 3, 64 cameras at
    1920x1080), forward passes only (projection, binning, sort, blend), the cameras split
    over the ranks (rank r renders cameras r, r + world, ...). Device-timed over
    `forward_batches` passes of the camera batch after one untimed pass; the value is every
    rank's pixels over the slowest rank's time."""
    import torch

    import splat_b200 as sb
    from splat_b200 import scenes

    scene = scenes.config(3)
    cams = scene.cameras[rank::world]
    w, h = cams[0].width, cams[0].height
    params = torch.from_numpy(scene.cloud.to_packed()).cuda()
    opts = sb.default_options(sh_degree=scene.cloud.sh_degree,
                              tile_culling=sb.SP_TILES_ELLIPSE if args.tiles == "ellipse" else sb.SP_TILES_RECTANGLE)
    rast = sb.Rasterizer(ctx, params, len(scene.cloud), w, h, None, 0, opts)
    uniforms = [c.uniform() for c in cams]

    def batch() -> None:
        for u in uniforms:
            rast.set_camera(u)
            rast.encode_forward()

    batch()
    meta = rast.read_intersections_unchecked()
    ctx.profile(True)
    batch()
    ctx.profile(False)
    profile = {k: v for k, v in ctx.read_profile().items() if v[1]}
    barrier()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.forward_batches):
        batch()
    stop.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(start.elapsed_time(stop))
    pixels = len(scene.cameras) * w * h * args.forward_batches
    out = {
        "value": pixels / (ms / 1000.0) / 1e6,
        "unit": "Mpix/s",
        "workload": f"config 3: {len(scene.cloud)} Gaussians SH{scene.cloud.sh_degree}, {len(scene.cameras)} cameras "
                    f"{w}x{h}, forward only, cameras split over {world} GPU(s)",
        "ms_per_view": ms / (len(scene.cameras) * args.forward_batches / world),
        "intersections_last_view": int(meta.count),
        "overflow": bool(meta.overflow),
        "kernels_ms_per_view": {k: v[0] / len(uniforms) for k, v in profile.items()},
    }
    rast.close()
    del params
    torch.cuda.empty_cache()
    return out


def main() -> None:
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
        return

    import torch
    import torch.distributed as dist

    import splat_b200 as sb
    from splat_b200 import scenes, sharding
    from splat_b200.sharding import ViewShardedStep

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=torch.device("cuda", local))

    scene = scenes.config(CONFIG_INDEX, scale=args.scale)
    if args.views:
        scene.cameras = scene.cameras[: args.views]
    cloud, cams = scene.cloud, scene.cameras
    deg = cloud.sh_degree
    views = len(cams)
    width, height = cams[0].width, cams[0].height
    ctx = sb.Context(local)
    culling = sb.SP_TILES_ELLIPSE if args.tiles == "ellipse" else sb.SP_TILES_RECTANGLE
    options = lambda: sb.default_options(sh_degree=deg, backward_mode=sb.SP_BWD_ATOMIC,  # noqa: E731
                                         tile_culling=culling)
    gt_host = build_ground_truth(ctx, scene, options)
    params = torch.from_numpy(cloud.to_packed()).cuda()
    initial = params.clone()
    gt = torch.from_numpy(gt_host.reshape(-1)).cuda()
    rast = sb.Rasterizer(ctx, params, len(cloud), width, height, gt, views, options())
    extent = np.float32(sb.cameras_extent(cams))
    adam = sb.Adam(ctx, params, rast, len(cloud), sb.LEARNING_RATES_3DGS, extent, sh_degree=deg)
    uniforms = [c.uniform() for c in cams]
    iterations = scene.iterations
    # One GPU: backward with the Adam step fused. N GPUs: gradients reduce-scattered, Adam on
    # this rank's share of the Gaussians, parameters all-gathered (splat_b200/sharding.py).
    exchange_mode = None if args.exchange == "auto" else args.exchange
    # N GPUs: the library's own communicator (sp_comm_*) carries the exchange; its id travels
    # from rank 0 through torch.distributed's object broadcast (plumbing only).
    comm = None
    if world > 1:
        from splat_b200.comm import Communicator

        uid = [Communicator.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        comm = Communicator(ctx, uid[0], world, rank, timeout_ms=180_000)
    train_step = ViewShardedStep(rast, adam, params, uniforms, rank, world, mode=exchange_mode, comm=comm)

    def view_of(step: int) -> int:
        return sharding.view_of(step, rank, world, views)

    def device_step(step: int) -> None:
        train_step(step, sb.position_rate_factor(step % iterations, iterations))

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for i in range(args.warmup):
        device_step(i)
    meta = rast.read_intersections_unchecked()

    # ---- per-kernel device time over one pass of every view (CUDA events on the
    # launching stream), then the blend work of those views, on the state the timed
    # region starts from.
    ctx.profile(True)
    for i in range(views):
        device_step(args.warmup + i)
    ctx.profile(False)
    profile = ctx.read_profile()
    # The blend kernels' algorithmic work is the reference's per-pixel loops over its lists (the
    # whole rectangles), counted on a rasterizer with the reference's lists even when the timed
    # one culls tiles by the ellipse (whose lists hold the same contributing entries).
    counter = rast if culling == sb.SP_TILES_RECTANGLE else sb.Rasterizer(
        ctx, params, len(cloud), width, height, gt, views,
        sb.default_options(sh_degree=deg, backward_mode=sb.SP_BWD_ATOMIC))
    fwd_pairs, bwd_pairs, taken_pairs = 0, 0, 0
    for v in range(views):
        counter.set_camera(uniforms[v])
        counter.encode_forward()
        f, b, t = counter.count_blend_work()
        fwd_pairs += f
        bwd_pairs += b
        taken_pairs += t
    if counter is not rast:
        counter.close()
        del counter
    first_timed = args.warmup + views

    # ---- value: device-resident throughput. The clock sampler is running before the ranks
    # meet at the barrier, so that no rank's start waits on it.
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier()
        start.record()
        for i in range(args.steps):
            device_step(first_timed + i)
        stop.record()
        torch.cuda.synchronize()
    ms = max_over_ranks(start.elapsed_time(stop))
    value = world * args.steps / (ms / 1000.0)
    clock_summary = clocks.summary()

    # ---- the NVLink peak the exchange is judged against: rank 0 times a plain peer copy to
    # the next GPU while the other ranks wait.
    nvlink = None
    if world > 1:
        barrier()
        if rank == 0:
            copy = peer_copy_gbs(local, local + 1)
            probe = None
            if getattr(train_step.exchange, "mode", None) == "peer":
                # The link as the exchange kernel uses it: SM loads from the next rank's buffer.
                size = min(256 << 20, len(cloud) * sb.param_stride(deg) * 4) // 16 * 16
                probe = train_step.exchange.probe_link(1, size)
            nvlink = {"gbs_per_direction": probe if probe else copy,
                      "peer_read_gbs": probe,
                      "copy_engine_gbs": copy,
                      "how": ("peer-read kernel of the exchange (sp_exchange_probe_link: float4 loads from rank 1's "
                              "gradient buffer, 4 in flight per thread, CUDA events) " if probe else "")
                             + f"and cudaMemcpyAsync (torch copy_) of 512 MiB from GPU {local} to GPU {local + 1}"}
        barrier()

    # ---- e2e: the reference caller's step through the public API, poses refined.
    params.copy_(initial)
    adam_e2e = sb.Adam(ctx, params, rast, len(cloud), sb.LEARNING_RATES_3DGS, extent, sh_degree=deg)
    exchange_e2e = sharding.make_exchange(adam_e2e, params, rast, rank, world, exchange_mode, comm=comm)
    poses = sb.PoseRefinement(cams, sb.LEARNING_RATES_3DGS, float(extent))
    e2e_steps = args.e2e_steps or args.steps

    def api_step(step: int) -> None:
        v = view_of(step)
        factor = sb.position_rate_factor(step % iterations, iterations)
        if world == 1:
            # One library call: the refinement's camera, the step, its 88-byte read-back and
            # the host pose step.
            rast.train_step_host_poses(adam_e2e, poses, v, factor)
            return
        else:
            rast.set_camera(poses.camera(v))
            rast.encode_forward()
            rast.encode_loss(v)
            rast.encode_backward()
            exchange_e2e(factor)
            gradient = rast.read_camera_gradient()
            rast.read_loss()
        poses.step(v, gradient, factor)

    for i in range(min(args.warmup, 3)):
        api_step(i)
    barrier()
    e_start, e_stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record()
    for i in range(e2e_steps):
        api_step(args.warmup + i)
    e_stop.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e_start.elapsed_time(e_stop))
    e2e_value = world * e2e_steps / (e2e_ms / 1000.0)

    # ---- e2e with the poses refined on the device (one GPU): the same steps through
    # sp_train_step_device_poses, no host synchronisation per step; each step's loss sums
    # (32 B) land in their own slot of a pinned host ring.
    e2e_device = None
    if world == 1:
        params.copy_(initial)
        adam_dp = sb.Adam(ctx, params, rast, len(cloud), sb.LEARNING_RATES_3DGS, extent, sh_degree=deg)
        device_poses = sb.DevicePoses(rast, sb.PoseRefinement(cams, sb.LEARNING_RATES_3DGS, float(extent)))
        ring = torch.zeros((64, 4), dtype=torch.float64).pin_memory()

        def device_pose_step(step: int) -> None:
            factor = sb.position_rate_factor(step % iterations, iterations)
            rast.train_step_device_poses(adam_dp, device_poses, view_of(step), view_of(step + 1), factor,
                                         ring[step % len(ring)])

        device_poses.set_camera(view_of(0))
        for i in range(min(args.warmup, 3)):
            device_pose_step(i)
        barrier()
        d_start, d_stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        d_start.record()
        for i in range(e2e_steps):
            device_pose_step(args.warmup + i)
        d_stop.record()
        torch.cuda.synchronize()
        device_poses.download()
        d_ms = d_start.elapsed_time(d_stop)
        e2e_device = {
            "value": e2e_steps / (d_ms / 1000.0),
            "unit": UNIT,
            "h2d_bytes_per_step": 0,
            "d2h_bytes_per_step": 32,
            "what": "sp_train_step_device_poses: forward + loss + backward + Adam + the pose step on the device, "
                    "the next view's camera written on the device, the loss sums (32 B) written into pinned "
                    "host memory by the loss-sum kernel; no host synchronisation per step",
        }
        device_poses.close()
        del adam_dp

    launches_per_step = sum(n for _, n in profile.values()) / views
    pk = peaks()
    fp32_peak = SMS * FP32_LANES_PER_SM * pk["sm_max_mhz"] * 1e6 / 1e12  # T FP32 instructions / s
    n_params = len(cloud) * sb.param_stride(deg)
    kernels = {}
    for name, (kms, n) in profile.items():
        if n == 0:
            continue
        entry = {"ms_per_launch": kms / n, "launches": n, "share": kms / max(sum(t for t, _ in profile.values()), 1e-9)}
        if name == "blend_forward":
            achieved = fwd_pairs / views * FORWARD_OPS_PER_PAIR / (kms / n * 1e-3) / 1e12
            entry.update(bound="fp32", achieved=achieved, peak=fp32_peak, unit="T FP32 ops/s",
                         frac=achieved / fp32_peak, pairs_per_launch=fwd_pairs / views,
                         # The pairs that blend (alpha >= 1/255 before the termination), of the
                         # reference's visited pairs the roofline counts.
                         active_pairs_per_launch=taken_pairs / views,
                         active_fraction=taken_pairs / max(fwd_pairs, 1))
        elif name == "blend_backward":
            achieved = bwd_pairs / views * BACKWARD_OPS_PER_PAIR / (kms / n * 1e-3) / 1e12
            entry.update(bound="fp32", achieved=achieved, peak=fp32_peak, unit="T FP32 ops/s",
                         frac=achieved / fp32_peak, pairs_per_launch=bwd_pairs / views,
                         active_pairs_per_launch=taken_pairs / views,
                         active_fraction=taken_pairs / max(bwd_pairs, 1))
        elif name == "adam":
            # The sharded exchange steps this rank's share of the Gaussians only.
            stepped = n_params // world if world > 1 and train_step.exchange.mode == "sharded" else n_params
            achieved = stepped * 28 / (kms / n * 1e-3) / 1e9
            entry.update(bound="hbm", achieved=achieved, peak=pk["hbm_gbs"], unit="GB/s", frac=achieved / pk["hbm_gbs"],
                         bytes_per_launch=stepped * 28)
        elif name == "peer_adam":
            # Per launch and link direction of this GPU: its reads of its share of the peers'
            # gradients and the peers' stores of their shares into it come in, its stores and
            # the peers' reads of its gradients go out: 2 (world - 1) shares each way, against
            # the peer copy measured above (rank 0), else the pool's recorded 770 GB/s.
            share_bytes = n_params // world * 4
            link_bytes = 2 * (world - 1) * share_bytes
            achieved = link_bytes / (kms / n * 1e-3) / 1e9
            link_peak = nvlink["gbs_per_direction"] if nvlink else 770.0
            entry.update(bound="nvlink", achieved=achieved, peak=link_peak, unit="GB/s per direction",
                         frac=achieved / link_peak, nvlink_bytes_per_direction=link_bytes,
                         hbm_bytes=share_bytes * (1 + 6),
                         peak_source=("measured peer copy (nvlink key)" if nvlink
                                      else "recorded peer copy of this pool, 770 GB/s per direction"))
        elif name == "backward_adam":
            # Parameters and both moments read and written, the 9 blend sums read.
            b = n_params * 24 + len(cloud) * 36
            achieved = b / (kms / n * 1e-3) / 1e9
            entry.update(bound="hbm", achieved=achieved, peak=pk["hbm_gbs"], unit="GB/s", frac=achieved / pk["hbm_gbs"],
                         bytes_per_launch=b)
        elif name == "project":
            # Parameters in; the 64-B blend record, 16-B culling constants, radius and tile count out.
            b = len(cloud) * (4 * sb.param_stride(deg) + 88)
            achieved = b / (kms / n * 1e-3) / 1e9
            entry.update(bound="hbm", achieved=achieved, peak=pk["hbm_gbs"], unit="GB/s", frac=achieved / pk["hbm_gbs"],
                         bytes_per_launch=b)
        kernels[name] = entry
    dominant = max(kernels, key=lambda k: kernels[k]["share"])
    d = kernels[dominant]
    roofline = {
        "kernel": dominant,
        "bound": d.get("bound"),
        "achieved": d.get("achieved"),
        "peak": d.get("peak"),
        "unit": d.get("unit"),
        "frac": d.get("frac"),
        "traffic": NCU_TRAFFIC_BYTES.get(dominant),
        "peak_source": ("nominal FP32 issue rate: 148 SMs x 128 lanes x sm_max clock (FMA = 1 op)"
                        if d.get("bound") == "fp32" else d.get("peak_source") if d.get("bound") == "nvlink"
                        else f"{pk['source']} HBM copy bandwidth (MEASURED_PEAKS.json)"),
    }

    densify = None
    if world == 1 and not args.no_densify:
        densify = densify_timing(ctx, train_step.rasterizer, train_step.adam, float(extent), len(cloud))

    web_example = None
    if world == 1 and not args.no_web_example:
        web_example = web_example_timing(ctx)

    config5 = None
    if not args.no_config5:
        config5 = config5_throughput(args, ctx, comm, rank, world, max_over_ranks, barrier)

    forward_3m = None
    if not args.no_forward_3m:
        forward_3m = forward_throughput(args, ctx, rank, world, max_over_ranks, barrier)

    baseline = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        baseline = cpu_baseline(scene, gt_host, args.cpu_seconds)
        baseline.pop("ms_per_step", None)
        baseline.pop("steps", None)
        if densify is not None:
            # The reference's densification of the same state: read back, then densify on the host.
            r, a = train_step.rasterizer, train_step.adam
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            host_params = train_step.params.cpu().numpy()
            first, second = a.read_moments()
            stats = r.read_densify_stats()
            readback_ms = 1000.0 * (time.perf_counter() - t0)
            baseline["densify"] = cpu_densify(host_params, first, second, stats, r.stride, float(extent),
                                              sb.DENSIFY_SHORT_RUN.max_count(len(cloud)), sb.DENSIFY_SHORT_RUN)
            baseline["densify"]["readback_ms"] = readback_ms

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": value,
            "unit": UNIT,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms / args.steps,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f32",
            "data": "synthetic",
            "config": config_dict(scene, world, train_step.exchange.mode),
            "tile_culling": (f"{args.tiles}: " + (
                "keys only for the bounding rectangle's tiles the Gaussian's alpha can reach (the same images, "
                "losses and gradients as the reference's whole rectangles)"
                if args.tiles == "ellipse" else "the reference's whole bounding rectangles")),
            "clocks": clock_summary,
            "nvlink": nvlink,
            "libraries_loaded": libraries_loaded(),
            "e2e": {
                "value": e2e_value,
                "unit": UNIT,
                "h2d_bytes_per_step": 80,
                "d2h_bytes_per_step": 96 if world == 1 else 56 + 32,
                "what": "set_camera (80-B camera uniform from the host) + forward + loss + backward + Adam, then the "
                        "camera gradient (56 B), the step status and the loss sums (32 B) read back (one 96-B copy "
                        "on one GPU) and the host pose step",
            },
            "e2e_device_poses": e2e_device,
            "gpu_launches": int(round(launches_per_step * args.steps)),
            "roofline": roofline,
            "cpu_baseline": baseline,
            "kernels": kernels,
            "intersections": int(meta.count),
            "mpix_per_s": value * width * height / 1e6,
            "fwd_mpix_per_s_3M": forward_3m,
            "web_example": web_example,
            "config5": config5,
            "densify": densify,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        # Every rank's last exchange ended with its closing all-reduce: no peer access remains.
        torch.cuda.synchronize()
        dist.barrier()
        train_step.exchange.close()
        exchange_e2e.close()
        comm.close()
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
