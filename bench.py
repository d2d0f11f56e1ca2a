#!/usr/bin/env python
"""Stage-1 2D gaussian image fitting benchmark (fits/s) on 1..8 B200, one process per GPU.

Workload (default ``single_large``): a 1024x768 RGB fp32 target made of 5,000 random anisotropic
gaussians + N(0, 0.01) noise, fitted with 50,000 gaussians, L2 loss, Adam lr 1e-2 with the cosine
schedule, 1,000 iterations. One step = one complete fit of one image per GPU (``--views V``: V
images fitted together in one engine; weak scaling: rank r fits its own images, seeds
1000 + r * V + v), followed for N > 1 by the one gather of fitted parameters to all ranks (NCCL).
``value`` = images fitted by all ranks / max-over-ranks device time. Other workloads
(``--workload``): ``batched_720p`` (1280x720, 70,000 gaussians, 1,000 iterations) and
``masked_540p`` (960x540, 30,000 gaussians initialised inside a binary ellipse-union mask, 600
iterations, L2 over the mask pixels read from bit-packed masks).

Also measured in the same run:
  e2e       the same fit through the public API (fit_image_from_initialization; several images:
            the batched fit; masked workloads: fit_views_batched_masked) with the targets, masks
            and initial parameters in pinned host memory and the fitted parameters read back.
  roofline  the fused raster kernel (forward + loss gradient + backward), timed with CUDA events
            on its launch stream around every raster launch of one extra fit of the same workload
            run right after the timed fits; algorithmic work = 68 FP32 flop per (gaussian,
            pixel-in-support-rectangle) pair.
  ranks     per-rank fit and gather device times of the timed steps and their spread (N > 1).
  sharded   the multi-view configurations through the product sharding API
            (distributed.fit_views_sharded): the 64 images of batched_720p and the 256 masked
            views of masked_540p split across the N ranks (strong scaling: total work fixed),
            images/s from the max-over-ranks device time, per-rank fit / gather times, and e2e
            with host images in and all fitted parameters back on the host.
  splat     the 4K micro-benchmark: 1,000,000 fixed gaussians on 3840x2160, forward + backward
            through the renderer C ABI with an N(0,1) upstream gradient (Gpixel.gauss/s), beside
            the CPU oracle's forward + backward on a 1/64 subset of the gaussians.
  single_small  the 128x128 / 2,000-gaussian / 200-iteration fit: on the GPU through the public
            API, and on the CPU with the oracle, timed in full (N = 1).
  cpu_baseline  the CPU oracle (restatement of the reference's pure-PyTorch fit) on the host
            cores: 5 timed iterations at the start, the middle and the end of the fit (parameter
            states taken from the GPU fit), combined by the trapezoid rule into fits/s.

``--impl reference`` times only that CPU implementation (rank 0; other ranks exit at once), on
the same workload and config: each step is 5 oracle iterations from the fit's initial state.
Every CPU timing renders with the reference's pair chunks (max(64 x width, 65536) pairs per
index_add, each into a new copy of the frame): that chunk size, not the arithmetic, sets much of
the reference's CPU time (the oracle's renders do not depend on it, its gradients only to float32
rounding).
"""

from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (str(ROOT), str(ROOT / "realtime-gs_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402
import torch  # noqa: E402

FLOP_PER_PAIR = 68.0  # 20 forward + 48 backward FP32 flop per pair (FMA = 2)
FP32_LANES = 148 * 128  # SMs x FP32 lanes per SM on B200


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("native", "reference"), default="native")
    ap.add_argument("--workload", default="single_large")
    ap.add_argument("--views", type=int, default=1,
                    help="images fitted together in one engine per GPU and step (batched fit); value counts images")
    ap.add_argument("--no-splat", action="store_true", help="skip the 4K splat micro-benchmark")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--no-sharded", action="store_true",
                    help="skip the multi-view configurations fitted through distributed.fit_views_sharded")
    ap.add_argument("--sharded-steps", type=int, default=2, help="timed passes of each sharded configuration")
    ap.add_argument("--iterations", type=int, default=None, help="override the fit length (profiling runs)")
    ap.add_argument("--no-e2e", action="store_true", help="skip the public-API end-to-end measurement")
    ap.add_argument("--only-splat", action="store_true", help="run only the 4K splat micro-benchmark")
    return ap.parse_args()


# ---------------------------------------------------------------------------------------------
def load_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text())
    return {"hbm_gbs": 6650.0, "sm_max_mhz": 1965.0, "fallback": True}


class ClockSampler:
    """nvidia-smi sampling of SM clock and throttle reasons while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, device: torch.device):
        self.proc = None
        self.file = None
        try:
            uuid = "GPU-" + str(torch.cuda.get_device_properties(device).uuid)
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-i", uuid, "-lms", "200"],
                stdout=self.file, stderr=subprocess.DEVNULL,
            )
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.file.flush()
        rows = []
        with open(self.file.name) as fh:
            for line in fh:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.file.name)
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        reasons = sorted({name for r in rows for name, v in zip(self.NAMES, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------------------------
CPU_SAMPLE_ITERS = 5  # oracle iterations timed per CPU sample (after one untimed iteration)


def workload_config(name: str, wl: dict, views: int, world: int) -> dict:
    """The ``config`` object of the JSON line: identical in the native and the reference arm."""
    return {
        "workload": name, "height": wl["height"], "width": wl["width"], "gaussians": wl["n_fit"],
        "iterations": wl["iterations"], "source_gaussians": wl["n_sources"],
        "source_sigma_px": list(wl["sigma"]), "noise_sd": wl["noise"],
        "images_per_gpu_per_step": views, "parallelism": f"dp{world} (whole images)",
        "loss": "L2 over mask pixels (bit-packed masks)" if wl.get("masked") else "L2",
        "l2": f"256 MB buffer written between timed fits; a fit's own {wl['iterations']} iterations run L2-warm",
    }


def orender_budget(wl: dict) -> int:
    """Pairs per index_add chunk of the reference's torch renderer at this workload's width."""
    from oracle import render2d as orender

    return orender.reference_budget(wl["width"])


def cpu_target(wl: dict, seed: int):
    """(target (H, W, 3), init (xy, chol, color, weight) stacked (1, N, .), mask (1, H, W) or None)
    of the workload on the CPU (oracle render of the sources)."""
    from oracle import render2d as orender
    from rtgs_b200.image2gs import synthetic

    h, w = wl["height"], wl["width"]
    src = synthetic.source_gaussians(seed, wl["n_sources"], h, w, wl["sigma"])
    with torch.no_grad():
        target = (orender.render(src.xy, src.chol, src.color, src.weight, h, w)
                  + synthetic.noise(seed, h, w, wl["noise"])).clamp(0, 1)
    mask = None
    if wl.get("masked"):
        mask = synthetic.ellipse_mask(seed, h, w)
        init = synthetic.masked_fit_init(seed, wl["n_fit"], mask)
        mask = mask[None]
    else:
        init = synthetic.fit_init(seed, wl["n_fit"], h, w)
    return target, tuple(x[None] for x in (init.xy, init.chol, init.color, init.weight)), mask


def oracle_seconds_per_iteration(target, state, wl: dict, mask, iters: int = CPU_SAMPLE_ITERS) -> float:
    """Seconds per iteration of the CPU oracle fit loop (build, render, loss, backward, Adam,
    cosine step) from parameter state ``state``: one untimed iteration, then ``iters`` timed."""
    from oracle import fit as ofit
    from oracle import render2d as orender

    fit = ofit.StackedFit(target[None], tuple(x.detach().cpu().clone() for x in state), wl["iterations"],
                          lr=1e-2, masks=mask, budget=orender.reference_budget(wl["width"]))
    fit.step(0)
    t0 = time.perf_counter()
    for it in range(1, iters + 1):
        fit.step(it)
    return (time.perf_counter() - t0) / iters


def cpu_fit_estimate(target, states: dict[int, tuple], wl: dict, mask) -> dict:
    """CPU oracle fits/s from timed samples at several points of the fit (iteration -> state):
    the seconds per iteration are integrated over the fit by the trapezoid rule."""
    torch.set_num_threads(os.cpu_count() or 1)
    points = sorted(states)
    sec = {k: oracle_seconds_per_iteration(target, states[k], wl, mask) for k in points}
    total = 0.0
    for a, b in zip(points[:-1], points[1:]):
        total += 0.5 * (sec[a] + sec[b]) * (b - a)
    total += sec[points[-1]] * (wl["iterations"] - points[-1])  # the last sample covers the tail
    total += sec[points[0]] * points[0]
    return {"value": 1.0 / total, "unit": "fits/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{wl['height']}x{wl['width']}, {wl['n_fit']} gaussians: {CPU_SAMPLE_ITERS} oracle iterations "
                      f"(after 1 untimed) from the parameter states at iterations {points} of the GPU fit, "
                      f"seconds per iteration integrated over the {wl['iterations']} iterations (trapezoid); "
                      f"the reference's {orender_budget(wl)}-pair index_add chunks",
            "s_per_iteration_at": {str(k): sec[k] for k in points},
            "start_of_fit_value": 1.0 / (sec[points[0]] * wl["iterations"])}


def run_reference(args, wl, rank: int, world: int) -> None:
    """The reference arm: the CPU oracle alone, each step CPU_SAMPLE_ITERS iterations from the fit's
    initial state (no GPU involved), scaled to the fit's iteration count."""
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    target, init, mask = cpu_target(wl, 1000)
    for _ in range(args.warmup):
        oracle_seconds_per_iteration(target, init, wl, mask, iters=1)
    per_iter = [oracle_seconds_per_iteration(target, init, wl, mask) for _ in range(args.steps)]
    sec = statistics.median(per_iter)
    value = 1.0 / (sec * wl["iterations"])
    line = {
        "metric": "2D-gaussian image fits/sec", "value": value, "unit": "fits/s", "impl": "reference",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": sec * CPU_SAMPLE_ITERS * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(args.workload, wl, max(1, int(args.views)), world),
        "cpu_baseline": {"value": value, "unit": "fits/s", "cores": torch.get_num_threads(), "kind": "port",
                         "sample": f"each step: {CPU_SAMPLE_ITERS} oracle iterations (after 1 untimed) from the "
                                   f"fit's initial state, {wl['height']}x{wl['width']}, {wl['n_fit']} gaussians; "
                                   f"median of {args.steps} steps scaled to {wl['iterations']} iterations; "
                                   f"the reference's {orender_budget(wl)}-pair index_add chunks"},
        "e2e": {"value": value, "unit": "fits/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def cpu_splat_sample(stride: int = 64) -> dict:
    """CPU oracle forward + backward of the 4K splat on every ``stride``-th gaussian (same upstream
    gradient, the reference's pair chunks); throughput in (gaussian, pixel-in-rectangle) pairs per
    second. The chunk count grows with the pairs, so the rate does not depend on the stride."""
    from oracle import render2d as orender
    from rtgs_b200.image2gs import synthetic

    torch.set_num_threads(os.cpu_count() or 1)
    h, w = 2160, 3840
    sc = synthetic.splat_scene(0)
    sub = [x[::stride][None].clone().requires_grad_(True) for x in (sc.xy, sc.chol, sc.color, sc.weight)]
    up = synthetic.splat_upstream_grad(0, 1, h, w)
    rects = orender.cuda_rects(sub[0][0].detach(), sub[1][0].detach(), h, w)
    pairs = orender.pair_count(rects, torch.isfinite(sub[0][0].detach()).all(1))
    t0 = time.perf_counter()
    img = orender.render_batched(*sub, h, w, budget=orender.reference_budget(w))
    (img * up).sum().backward()
    dt = time.perf_counter() - t0
    return {"gpairs_per_s": pairs / dt / 1e9, "pairs": pairs, "s": dt, "cores": torch.get_num_threads(),
            "sample": f"one forward + backward of every {stride}th gaussian ({sub[0].shape[1]} of 1,000,000) "
                      f"on the 3840x2160 frame, oracle renderer with the reference's "
                      f"{orender.reference_budget(w)}-pair index_add chunks"}


def single_small_block(device) -> dict:
    """The 128x128 / 2,000-gaussian / 200-iteration fit: GPU (device-timed engine fits and the public
    API on host buffers) and the CPU oracle, each timed in full."""
    from oracle import fit as ofit
    from rtgs_b200.core.gaussians2d import Gaussians2D
    from rtgs_b200.image2gs import synthetic
    from rtgs_b200.image2gs.fit import FitConfig, fit_image_from_initialization

    wl = synthetic.WORKLOADS["single_small"]
    target, init, _ = cpu_target(wl, 0)
    cfg = FitConfig(n_gaussians=wl["n_fit"], iterations=wl["iterations"], log_every=50)
    host = [target.pin_memory()] + [x[0].pin_memory() for x in init]
    times = []
    for k in range(4):
        torch.cuda.synchronize(device)
        t0 = time.perf_counter()
        dev = [x.to(device, non_blocking=True) for x in host]
        fitted, hist = fit_image_from_initialization(dev[0], Gaussians2D(*dev[1:]), cfg)
        out = fitted.xy.cpu(), fitted.chol.cpu(), fitted.color.cpu(), fitted.weight.cpu()
        torch.cuda.synchronize(device)
        if k > 0:
            times.append(time.perf_counter() - t0)
    torch.set_num_threads(os.cpu_count() or 1)
    budget = orender_budget(wl)
    t0 = time.perf_counter()
    _, ohist = ofit.fit_views(target[None], init, wl["iterations"], lr=1e-2, log_every=50, budget=budget)
    cpu_s = time.perf_counter() - t0
    e2e = 1.0 / statistics.median(times)
    return {"workload": "single_small: 128x128, 500 sources, 2,000 gaussians, 200 iterations",
            "e2e_fits_per_s": e2e, "api": "fit_image_from_initialization (host buffers in and out)",
            "cpu_fits_per_s": 1.0 / cpu_s, "cpu_cores": torch.get_num_threads(),
            "cpu_sample": "one complete oracle fit (200 iterations + final render), kind port, with the "
                          f"reference's {budget}-pair index_add chunks",
            "e2e_vs_cpu": e2e * cpu_s, "final_psnr_gpu": hist["final_psnr"],
            "final_psnr_cpu": ohist[0]["final_psnr"]}


# ---------------------------------------------------------------------------------------------
def splat_microbench(device, steps: int, warmup: int) -> dict:
    """4K frame, 1M fixed gaussians: forward + backward through the renderer C ABI."""
    from rtgs_b200 import _native
    from rtgs_b200.image2gs import synthetic

    h, w = 2160, 3840
    sc = synthetic.splat_scene(0, n=1_000_000, height=h, width=w)
    xy, chol, color, weight = (x.to(device).contiguous() for x in (sc.xy, sc.chol, sc.color, sc.weight))
    up = synthetic.splat_upstream_grad(0, 1, h, w).to(device)
    out = torch.empty(1, h, w, 3, device=device)
    grads = [torch.empty_like(x) for x in (xy, chol, color, weight)]
    lib = _native.lib()
    arena = _native.arena(device)
    stream = _native.stream_ptr(device)
    m = xy.shape[0]

    def step(mid=None):
        _native.check(lib.rtgs2d_render_forward(arena, xy.data_ptr(), chol.data_ptr(), color.data_ptr(),
                                                weight.data_ptr(), 1, m, h, w, out.data_ptr(), None, stream))
        if mid is not None:
            mid.record()
        # The backward of an autograd step: it reuses the forward's projection and binning.
        _native.check(lib.rtgs2d_render_backward_after_forward(
            arena, up.data_ptr(), None, xy.data_ptr(), chol.data_ptr(), color.data_ptr(), weight.data_ptr(),
            1, m, h, w, *(g.data_ptr() for g in grads), stream))

    for _ in range(warmup):
        step()
    torch.cuda.synchronize(device)
    times, fwd = [], []
    for _ in range(steps):
        e0, em, e1 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record()
        step(em)
        e1.record()
        e1.synchronize()
        times.append(e0.elapsed_time(e1))
        fwd.append(e0.elapsed_time(em))
    entries, pairs = _native.arena_last_stats(device)
    ms = statistics.median(times)
    fwd_ms = statistics.median(fwd)
    return {"pairs": pairs, "entries": entries, "ms": ms, "forward_ms": fwd_ms, "backward_ms": ms - fwd_ms,
            "gpairs_per_s": pairs / (ms * 1e-3) / 1e9}


def e2e_fit(device, wl, targets_host, init_host, masks_host, steps: int) -> tuple[float, int, int, str]:
    """Public-API fit of the rank's images with host inputs.

    One image without a mask: ``fit_image_from_initialization``; several images: the batched fit
    (``fit_stacked``, the engine call behind ``fit_views_batched``); masked images:
    ``fit_views_batched_masked`` with boolean masks. Returns (median seconds per step, h2d bytes,
    d2h bytes, API name).
    """
    from rtgs_b200.core.gaussians2d import Gaussians2D
    from rtgs_b200.image2gs.batched import fit_stacked, fit_views_batched_masked
    from rtgs_b200.image2gs.fit import FitConfig, fit_image_from_initialization

    views = targets_host.shape[0]
    cfg = FitConfig(n_gaussians=wl["n_fit"], iterations=wl["iterations"], log_every=50)
    h2d = targets_host.numel() * 4 + sum(x.numel() * 4 for x in init_host)
    if masks_host is not None:
        h2d += masks_host.numel() * masks_host.element_size()
        api = "fit_views_batched_masked"
    else:
        api = "fit_image_from_initialization" if views == 1 else "fit_stacked (fit_views_batched)"
    times = []
    # Fitted parameters come back into pinned host buffers (asynchronous copies, one wait).
    out = [torch.empty(x.shape, dtype=torch.float32, pin_memory=True) for x in init_host]
    d2h = sum(x.numel() * 4 for x in out)
    warmup = 2  # the first call creates the pooled engine; the second reuses it once
    for k in range(steps + warmup):
        torch.cuda.synchronize(device)
        t0 = time.perf_counter()
        images = targets_host.to(device, non_blocking=True)
        init = tuple(x.to(device, non_blocking=True) for x in init_host)
        if masks_host is not None:
            masks = masks_host.to(device, non_blocking=True)
            fitted, _hist = fit_views_batched_masked(list(images), list(masks), init, cfg)
        elif views == 1:
            fitted, _hist = fit_image_from_initialization(images[0], Gaussians2D(*(x[0] for x in init)), cfg)
            fitted = [fitted]
        else:
            fitted, _hist = fit_stacked(images, init, cfg)
        for i, dst in enumerate(out):
            src = torch.stack([(g.xy, g.chol, g.color, g.weight)[i] for g in fitted])
            dst.copy_(src, non_blocking=True)
        torch.cuda.synchronize(device)
        dt = time.perf_counter() - t0
        if k >= warmup:
            times.append(dt)
    return statistics.median(times), h2d, d2h, api


def gather_floats(values: list[float], world: int) -> list[list[float]]:
    """Every rank's list of floats (host objects through the process group); [values] at N = 1."""
    if world == 1:
        return [list(values)]
    import torch.distributed as dist

    out: list = [None] * world
    dist.all_gather_object(out, list(values))
    return out


def max_over_ranks(value: float, device, world: int) -> float:
    t = torch.tensor([value], dtype=torch.float64, device=device)
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


SHARDED_ENGINE_VIEWS = {"batched_720p": 8, "masked_540p": 32}


def sharded_block(name: str, device, rank: int, world: int, steps: int, warmup: int) -> dict:
    """All views of multi-view workload `name` fitted through distributed.fit_views_sharded: rank r
    fits its contiguous block (the views of one engine at a time), then every rank gathers every
    view's fitted parameters. Strong scaling: the total number of views is fixed."""
    from rtgs_b200.image2gs import synthetic
    from rtgs_b200.image2gs.batched import fit_stacked
    from rtgs_b200.image2gs.distributed import fit_views_sharded, shard_range
    from rtgs_b200.image2gs.fit import FitConfig
    from rtgs_b200.image2gs.renderer2d import render_gaussians_2d_batched

    wl = synthetic.WORKLOADS[name]
    n_images, h, w, n = wl["n_views"], wl["height"], wl["width"], wl["n_fit"]
    masked = bool(wl.get("masked"))
    per_engine = SHARDED_ENGINE_VIEWS[name]
    base_seed = 2000  # view i uses seed 2000 + i whatever the number of ranks
    start, stop = shard_range(n_images, rank, world)
    seeds = list(range(base_seed + start, base_seed + stop))
    targets = [synthetic.make_target(sd, wl, render_gaussians_2d_batched, device) for sd in seeds]
    masks = [synthetic.ellipse_mask(sd, h, w) for sd in seeds] if masked else None
    inits = [synthetic.masked_fit_init(sd, n, m) if masked else synthetic.fit_init(sd, n, h, w)
             for sd, m in zip(seeds, masks or [None] * len(seeds))]
    init_rows = [(g.xy, g.chol, g.color, g.weight) for g in inits]
    cfg = FitConfig(n_gaussians=n, iterations=wl["iterations"], log_every=50)
    fit_end: list = []

    def fit_fn(local, config, first_seed):
        results, hists = [], []
        for b0 in range(0, len(local), per_engine):
            b1 = min(b0 + per_engine, len(local))
            imgs = torch.stack([im.to(device, non_blocking=True) for im in local[b0:b1]])
            init = tuple(torch.stack([row[k] for row in init_rows[b0:b1]]).to(device, non_blocking=True)
                         for k in range(4))
            m = torch.stack(masks[b0:b1]).to(device, non_blocking=True) if masked else None
            r, hh = fit_stacked(imgs, init, config, masks=m)
            results += r
            hists += hh
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        fit_end.append(ev)
        return results, hists

    def run(images):
        return fit_views_sharded(images, cfg, base_seed, fit_fn=fit_fn, device=device)

    images = [None] * n_images
    images[start:stop] = targets
    for _ in range(warmup):
        run(images)
    torch.cuda.synchronize(device)
    fit_ms, gather_ms, total_ms = [], [], []
    psnr = []
    for _ in range(steps):
        barrier(world)
        torch.cuda.synchronize(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        _, hist = run(images)
        e1.record()
        e1.synchronize()
        total_ms.append(e0.elapsed_time(e1))
        fit_ms.append(e0.elapsed_time(fit_end[-1]))
        gather_ms.append(total_ms[-1] - fit_ms[-1])
        psnr = [hh["final_psnr"] for hh in hist]
    step_ms = max_over_ranks(statistics.median(total_ms), device, world)
    # e2e: host images (and host masks / initial parameters) in, every view's parameters out
    host_images = [None] * n_images
    host_images[start:stop] = [t.cpu().pin_memory() for t in targets]
    init_rows = [tuple(x.pin_memory() for x in row) for row in init_rows]
    if masked:
        masks = [m.pin_memory() for m in masks]
    out_host = torch.empty(n_images, n, 9, pin_memory=True)
    e2e_runs = []
    for _ in range(steps):  # median over as many runs as the device timing
        barrier(world)
        torch.cuda.synchronize(device)
        t0 = time.perf_counter()
        fitted, _ = run(host_images)
        packed = torch.stack([torch.cat([g.xy, g.chol, g.color, g.weight[:, None]], 1) for g in fitted])
        out_host.copy_(packed, non_blocking=True)
        torch.cuda.synchronize(device)
        e2e_runs.append(time.perf_counter() - t0)
    e2e_s = max_over_ranks(statistics.median(e2e_runs), device, world)
    ranks_fit = gather_floats([statistics.median(fit_ms)], world)
    ranks_gather = gather_floats([statistics.median(gather_ms)], world)
    fits = [r[0] for r in ranks_fit]
    h2d = sum(t.numel() * 4 for t in targets) + sum(x.numel() * 4 for row in init_rows for x in row)
    if masked:
        h2d += sum(m.numel() * m.element_size() for m in masks)
    return {
        "workload": f"{name}: {n_images} views of {w}x{h}, {n} gaussians each, {wl['iterations']} iterations"
                    + (", L2 over bit-packed ellipse masks" if masked else "")
                    + f"; views split {n_images}/{world} per GPU through distributed.fit_views_sharded "
                      f"({per_engine} views per engine), then one all-gather of every view's parameters",
        "scaling": "strong", "value": n_images / (step_ms / 1e3), "unit": "images/s",
        "ms_per_step": step_ms, "steps": steps, "warmup": warmup,
        "rank_fit_ms": fits, "rank_gather_ms": [r[0] for r in ranks_gather],
        "rank_fit_skew_ms": max(fits) - min(fits),
        "e2e": {"value": n_images / e2e_s, "unit": "images/s", "h2d_bytes_per_step": int(max_over_ranks(h2d, device, world) * world),
                "d2h_bytes_per_step": int(out_host.numel() * 4 * world),
                "api": "distributed.fit_views_sharded with host images"},
        "mean_final_psnr_db_rank0_views": float(np.mean(psnr)) if psnr else None,
    }


def run_native(args, wl, rank: int, world: int, local_rank: int) -> None:
    import torch.distributed as dist

    from rtgs_b200.image2gs import synthetic
    from rtgs_b200 import _native
    from rtgs_b200.image2gs.engine import FitEngine, pack_mask_bits
    from rtgs_b200.image2gs.fit import raw_from_gaussians
    from rtgs_b200.image2gs.renderer2d import render_gaussians_2d_batched

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    if args.only_splat:
        res = splat_microbench(device, steps=args.steps, warmup=args.warmup)
        if rank == 0:
            print(json.dumps({"splat_fwd_bwd": res}), flush=True)
        return
    h, w, n, iters = wl["height"], wl["width"], wl["n_fit"], wl["iterations"]
    views = max(1, int(args.views))
    masked = bool(wl.get("masked"))
    # Image v of rank r is global image r * views + v (its seeds do not depend on the GPU count).
    seeds = [1000 + rank * views + v for v in range(views)]
    targets = torch.stack([synthetic.make_target(sd, wl, render_gaussians_2d_batched, device) for sd in seeds])
    masks = None
    if masked:  # binary ellipse-union masks, loss restricted to them, means initialised inside them
        masks = torch.stack([synthetic.ellipse_mask(sd, h, w) for sd in seeds])
        inits = [synthetic.masked_fit_init(sd, n, m) for sd, m in zip(seeds, masks)]
    else:
        inits = [synthetic.fit_init(sd, n, h, w) for sd in seeds]
    init_stack = tuple(torch.stack([getattr(g, f) for g in inits]) for f in ("xy", "chol", "color", "weight"))
    init_dev = tuple(x.to(device) for x in init_stack)
    raw = {k: v.contiguous() for k, v in raw_from_gaussians(*init_dev, h, w).items()}
    engine = FitEngine(views, n, h, w, lr=1e-2, iterations=iters, log_every=50, device=device,
                       loss_mode=_native.LOSS_MASK_ONLY if masked else _native.LOSS_MSE)
    engine.set_targets(targets, pack_mask_bits(masks.to(device)) if masked else None)
    mask_px = (masks.reshape(views, -1) > 0.5).sum(1).double().numpy() if masked else np.full(views, float(h * w))
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=device)  # > 126 MB L2
    gathered = torch.empty(world, views * n, 9, device=device) if world > 1 else None
    fit_done = [None]

    def one_fit():
        engine.set_raw(raw)
        engine.run(iters)
        if world > 1:  # the single collective of the job: gather every rank's fitted parameters
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            fit_done[0] = ev
            xy, chol, color, weight = (t.reshape(views * n, -1) for t in engine.params())
            packed = torch.cat([xy, chol, color, weight], dim=1).contiguous()
            dist.all_gather_into_tensor(gathered, packed)

    for _ in range(args.warmup):
        one_fit()
    torch.cuda.synchronize(device)
    barrier(world)
    sampler = ClockSampler(device)
    step_ms, fit_ms = [], []
    t_wall = time.perf_counter()
    for _ in range(args.steps):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        one_fit()
        e1.record()
        e1.synchronize()
        step_ms.append(e0.elapsed_time(e1))
        fit_ms.append(e0.elapsed_time(fit_done[0]) if world > 1 else step_ms[-1])
    torch.cuda.synchronize(device)
    barrier(world)
    wall_s = time.perf_counter() - t_wall
    clocks = sampler.stop()
    _, sums = engine.evaluate(want_render=False)
    final_psnr = float(np.mean([-10.0 * math.log10(max(sums[b, 1] / (3.0 * mask_px[b]), 1e-12)) for b in range(views)]))
    # Stage split and the raster kernel's duration: one more fit of the same workload with CUDA
    # events around every stage of every iteration (recorded inside the replayed graphs). Kept out
    # of the timed fits because the event records themselves lengthen an iteration.
    engine.set_profiling(True)
    flush.zero_()
    engine.set_raw(raw)
    engine.run(iters)
    torch.cuda.synchronize(device)
    stages = engine.stage_times()
    engine.set_profiling(False)
    # Parameter states for the CPU baseline's samples (start, middle and end of the fit).
    cpu_states = {}
    if world == 1 and not args.no_cpu and views == 1:
        engine.set_raw(raw)
        cpu_states[0] = tuple(x[:1].cpu() for x in init_stack)
        for at in (iters // 2, iters - CPU_SAMPLE_ITERS - 1):
            engine.run(at - engine.stats()["step"])
            cpu_states[at] = tuple(x[:1].cpu() for x in engine.params())

    total_ms = max_over_ranks(sum(step_ms), device, world)
    value = world * views * args.steps / (total_ms / 1e3)
    ranks_fit = [r[0] for r in gather_floats([statistics.median(fit_ms)], world)]
    ranks_step = [r[0] for r in gather_floats([statistics.median(step_ms)], world)]

    # e2e through the public API with host buffers (all ranks concurrently).
    targets_host = targets.cpu().pin_memory()
    init_host = tuple(x.pin_memory() for x in init_stack)
    masks_host = (masks > 0.5).pin_memory() if masked else None
    del engine
    e2e_value, h2d, d2h, e2e_api = None, 0, 0, None
    if not args.no_e2e:
        e2e_s, h2d, d2h, e2e_api = e2e_fit(device, wl, targets_host, init_host, masks_host, steps=5)
        e2e_value = world * views / max_over_ranks(e2e_s, device, world)

    sharded = {}
    if not args.no_sharded:
        for name in ("batched_720p", "masked_540p"):
            sharded[name] = sharded_block(name, device, rank, world, steps=args.sharded_steps, warmup=1)

    splat = None
    if not args.no_splat:
        splat = splat_microbench(device, steps=5, warmup=3)
        st = max_over_ranks(splat["ms"], device, world)
        splat["aggregate_gpairs_per_s"] = world * splat["pairs"] / (st * 1e-3) / 1e9

    if rank != 0:
        return
    peaks = load_peaks()
    sm_max = float(peaks.get("sm_max_mhz", 1965.0))
    fp32_peak = FP32_LANES * 2 * sm_max * 1e6 / 1e12  # TFLOP/s at the measured max SM clock
    raster_s = stages["raster_ms"] / 1e3
    achieved = FLOP_PER_PAIR * stages["pairs"] / raster_s / 1e12 if raster_s > 0 else None
    its = max(stages["iterations"], 1)
    traffic = None
    prof = ROOT / "profiles" / "raster_fit_single_large.json"
    if prof.exists():
        traffic = json.loads(prof.read_text()).get("dram_bytes_per_launch")
    cpu = None
    small = None
    cpu_splat = None
    if world == 1 and not args.no_cpu:
        if cpu_states:
            target_cpu = targets[0].cpu()
            res = cpu_fit_estimate(target_cpu, cpu_states, wl, masks[:1] if masked else None)
            cpu = {k: res[k] for k in ("value", "unit", "cores", "kind", "sample", "s_per_iteration_at",
                                       "start_of_fit_value")}
        small = single_small_block(device)
        if splat is not None:
            cpu_splat = cpu_splat_sample()
    # Own kernels per fit, per 64-iteration chunk of c iterations: the chunk's projection; the
    # first iteration's tile-count scan (own single-block kernel up to 8192 tiles, else CUB's two,
    # counted as library launches), scatter and tile sort; then per iteration raster fit (which
    # sorts its own tile's list after the first iteration) and Adam (+ the next projection with
    # direct placement), and for all but the last the next segment layout and tile order:
    # 3c + 3 own launches (3c + 2 plus 2 library ones above 8192 tiles).
    chunk_lens = [64] * (iters // 64) + ([iters % 64] if iters % 64 else [])
    n_tiles = views * ((h + 15) // 16) * ((w + 15) // 16)
    small_scan = n_tiles <= 8192
    own_per_fit = sum(3 * c + (3 if small_scan else 2) for c in chunk_lens)
    lib_per_fit = 0 if small_scan else 2 * len(chunk_lens)
    line = {
        "metric": "2D-gaussian image fits/sec",
        "value": value,
        "unit": "fits/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": total_ms / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": workload_config(args.workload, wl, views, world),
        "final_psnr_db": final_psnr,
        "e2e": {"value": e2e_value, "unit": "fits/s", "h2d_bytes_per_step": int(h2d * world),
                "d2h_bytes_per_step": int(d2h * world), "api": e2e_api},
        "roofline": {
            "bound": "fp32", "kernel": "raster_kernel<2,kFit> (fused forward + L2 gradient + backward)",
            "achieved": achieved, "peak": fp32_peak, "unit": "TFLOP/s",
            "frac": (achieved / fp32_peak) if achieved else None, "traffic": traffic,
            "peak_note": "148 SM x 128 FP32 lanes x 2 x measured max SM clock (MEASURED_PEAKS.json sm_max_mhz)",
            "flop_per_pair": FLOP_PER_PAIR, "pairs_per_launch": stages["pairs"] / its,
            "ms_per_launch": stages["raster_ms"] / its,
            "launch_timing": "CUDA events around every raster launch of one extra fit of this workload, "
                             "run right after the timed fits",
            "stage_ms_per_iteration": {"project_bin": stages["bin_ms"] / its, "raster": stages["raster_ms"] / its,
                                       "adam": stages["adam_ms"] / its},
        },
        "ranks": {"step_ms": ranks_step, "fit_ms": ranks_fit,
                  "gather_ms": [a - b for a, b in zip(ranks_step, ranks_fit)],
                  "fit_skew_ms": max(ranks_fit) - min(ranks_fit),
                  "note": "median over the timed steps per rank; step = fit + the parameter all-gather, "
                          "which waits for the slowest rank (each rank fits a different image)"},
        "cpu_baseline": cpu,
        "gpu_launches": args.steps * own_per_fit,
        "library_launches": args.steps * lib_per_fit,
        "clocks": clocks,
        "wall_s_timed_region": wall_s,
    }
    if sharded:
        line["sharded"] = sharded
    if small is not None:
        line["single_small"] = small
    if splat is not None:
        line["splat_fwd_bwd"] = {
            "workload": "splat_4k: 3840x2160, 1,000,000 gaussians, fixed parameters, N(0,1) upstream grad",
            "value": splat["aggregate_gpairs_per_s"], "unit": "Gpixel.gauss/s", "ms": splat["ms"],
            "forward_ms": splat["forward_ms"], "backward_ms": splat["backward_ms"],
            "pairs": splat["pairs"], "entries": splat["entries"],
            "achieved_tflops": FLOP_PER_PAIR * splat["pairs"] / (splat["ms"] * 1e-3) / 1e12,
            "frac_fp32": FLOP_PER_PAIR * splat["pairs"] / (splat["ms"] * 1e-3) / 1e12 / fp32_peak,
        }
        if cpu_splat is not None:
            line["splat_fwd_bwd"]["cpu_baseline"] = cpu_splat
    print(json.dumps(line), flush=True)


def main() -> None:
    args = parse_args()
    from rtgs_b200.image2gs.synthetic import WORKLOADS

    if args.workload not in WORKLOADS:
        raise SystemExit(f"unknown workload {args.workload}; choose from {sorted(WORKLOADS)}")
    wl = dict(WORKLOADS[args.workload])
    if args.iterations:
        wl["iterations"] = int(args.iterations)
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        run_reference(args, wl, rank, world)
        return
    if world > 1:
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_native(args, wl, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
