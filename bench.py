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
  splat     the 4K micro-benchmark: 1,000,000 fixed gaussians on 3840x2160, forward + backward
            through the renderer C ABI with an N(0,1) upstream gradient (Gpixel.gauss/s).
  cpu_baseline  the CPU oracle (restatement of the reference's pure-PyTorch fit) on the host
            cores, a bounded number of iterations of the same workload, scaled to fits/s.

``--impl reference`` times only that CPU implementation (rank 0; other ranks exit at once).
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
    ap.add_argument("--cpu-iters", type=int, default=2, help="oracle iterations per CPU sample step")
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
def cpu_fit_sample(wl: dict, seed: int, iters: int, steps: int, warmup: int) -> dict:
    """Time the CPU oracle fit (reference algorithm on torch CPU) for `iters` iterations per step."""
    from oracle import fit as ofit
    from oracle import render2d as orender
    from rtgs_b200.image2gs import synthetic

    torch.set_num_threads(os.cpu_count() or 1)
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
    init = tuple(x[None] for x in (init.xy, init.chol, init.color, init.weight))
    times = []
    for k in range(warmup + steps):
        t0 = time.perf_counter()
        ofit.fit_views(target[None], init, iters, lr=1e-2, log_every=10**9, masks=mask)
        dt = time.perf_counter() - t0
        if k >= warmup:
            times.append(dt)
    # fit_views also renders the final state once: subtract nothing (conservative for the CPU).
    per_iter = statistics.median(times) / (iters + 1)
    fits_per_s = 1.0 / (per_iter * wl["iterations"])
    return {"value": fits_per_s, "unit": "fits/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{wl['height']}x{wl['width']} target{' (masked loss)' if mask is not None else ''}, "
                      f"{wl['n_fit']} gaussians: {iters} oracle iterations "
                      f"(+1 final render) per step, median of {steps} steps after {warmup} warm-up, "
                      f"scaled to {wl['iterations']} iterations",
            "s_per_iteration": per_iter}


def run_reference(args, wl, rank: int) -> None:
    if rank != 0:
        return
    res = cpu_fit_sample(wl, 1000, args.cpu_iters, args.steps, args.warmup)
    line = {
        "metric": "2D-gaussian image fits/sec", "value": res["value"], "unit": "fits/s", "impl": "reference",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": res["s_per_iteration"] * args.cpu_iters * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.workload, **{k: v for k, v in wl.items() if k != "sigma"}, "sigma": list(wl["sigma"])},
        "cpu_baseline": {k: res[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": res["value"], "unit": "fits/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


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
    for k in range(steps + 1):
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
        if k > 0:  # the first call is a warm-up
            times.append(dt)
    return statistics.median(times), h2d, d2h, api


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

    def one_fit():
        engine.set_raw(raw)
        engine.run(iters)
        if world > 1:  # the single collective of the job: gather every rank's fitted parameters
            xy, chol, color, weight = (t.reshape(views * n, -1) for t in engine.params())
            packed = torch.cat([xy, chol, color, weight], dim=1).contiguous()
            dist.all_gather_into_tensor(gathered, packed)

    for _ in range(args.warmup):
        one_fit()
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    sampler = ClockSampler(device)
    step_ms = []
    t_wall = time.perf_counter()
    for _ in range(args.steps):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        one_fit()
        e1.record()
        e1.synchronize()
        step_ms.append(e0.elapsed_time(e1))
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    wall_s = time.perf_counter() - t_wall
    clocks = sampler.stop()
    _, sums = engine.evaluate(want_render=False)
    final_psnr = float(np.mean([-10.0 * math.log10(max(sums[b, 1] / (3.0 * mask_px[b]), 1e-12)) for b in range(views)]))
    # Stage split and the raster kernel's duration: one more fit of the same workload with CUDA
    # events around every stage of every iteration (recorded inside the replayed graphs). Kept out
    # of the timed fits because the event records themselves lengthen an iteration.
    engine.set_profiling(True)
    flush.zero_()
    one_fit()
    torch.cuda.synchronize(device)
    stages = engine.stage_times()
    engine.set_profiling(False)

    total_ms = torch.tensor([sum(step_ms)], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(total_ms, op=dist.ReduceOp.MAX)
    total_ms = float(total_ms.item())
    value = world * views * args.steps / (total_ms / 1e3)

    # e2e through the public API with host buffers (all ranks concurrently).
    targets_host = targets.cpu().pin_memory()
    init_host = tuple(x.pin_memory() for x in init_stack)
    masks_host = (masks > 0.5).pin_memory() if masked else None
    del engine
    e2e_value, h2d, d2h, e2e_api = None, 0, 0, None
    if not args.no_e2e:
        e2e_s, h2d, d2h, e2e_api = e2e_fit(device, wl, targets_host, init_host, masks_host, steps=2)
        e2e_t = torch.tensor([e2e_s], dtype=torch.float64, device=device)
        if world > 1:
            dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
        e2e_value = world * views / float(e2e_t.item())

    splat = None
    if not args.no_splat:
        splat = splat_microbench(device, steps=5, warmup=3)
        st = torch.tensor([splat["ms"]], dtype=torch.float64, device=device)
        if world > 1:
            dist.all_reduce(st, op=dist.ReduceOp.MAX)
        splat["aggregate_gpairs_per_s"] = world * splat["pairs"] / (float(st.item()) * 1e-3) / 1e9

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
    if world == 1 and not args.no_cpu:
        res = cpu_fit_sample(wl, seeds[0], args.cpu_iters, steps=1, warmup=1)
        cpu = {k: res[k] for k in ("value", "unit", "cores", "kind", "sample")}
    # Own kernels per fit, per 64-iteration chunk of c iterations: the chunk's projection; the
    # first iteration's tile-count scan (own single-block kernel up to 8192 tiles, else CUB's two,
    # counted as library launches) and scatter; then per iteration tile sort, raster fit and Adam
    # (+ the next projection), and for all but the last the next segment layout and tile order
    # (direct placement): 4c + 2 own launches (4c + 1 plus 2 library ones above 8192 tiles).
    chunk_lens = [64] * (iters // 64) + ([iters % 64] if iters % 64 else [])
    n_tiles = views * ((h + 15) // 16) * ((w + 15) // 16)
    small_scan = n_tiles <= 8192
    own_per_fit = sum(4 * c + (2 if small_scan else 1) for c in chunk_lens)
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
        "config": {
            "workload": args.workload, "height": h, "width": w, "gaussians": n, "iterations": iters,
            "source_gaussians": wl["n_sources"], "images_per_gpu_per_step": views, "parallelism": f"dp{world} (whole images)",
            "l2": f"256 MB buffer written between timed fits; a fit's own {iters} iterations run L2-warm",
            "loss": "L2 over mask pixels (bit-packed masks)" if masked else "L2",
            "final_psnr_db": final_psnr,
        },
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
        "cpu_baseline": cpu,
        "gpu_launches": args.steps * own_per_fit,
        "library_launches": args.steps * lib_per_fit,
        "clocks": clocks,
        "wall_s_timed_region": wall_s,
    }
    if splat is not None:
        line["splat_fwd_bwd"] = {
            "workload": "splat_4k: 3840x2160, 1,000,000 gaussians, fixed parameters, N(0,1) upstream grad",
            "value": splat["aggregate_gpairs_per_s"], "unit": "Gpixel.gauss/s", "ms": splat["ms"],
            "forward_ms": splat["forward_ms"], "backward_ms": splat["backward_ms"],
            "pairs": splat["pairs"], "entries": splat["entries"],
            "achieved_tflops": FLOP_PER_PAIR * splat["pairs"] / (splat["ms"] * 1e-3) / 1e12,
            "frac_fp32": FLOP_PER_PAIR * splat["pairs"] / (splat["ms"] * 1e-3) / 1e12 / fp32_peak,
        }
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
        run_reference(args, wl, rank)
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
