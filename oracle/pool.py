"""CPU oracle: the pooled (fixed-capacity, free-list) Stage-1 fit, restated from the reference.

TEST INFRASTRUCTURE ONLY -- imported by tests/, never by the product package.

Restated reference behaviour (paths relative to the reference project):
  - row store: capacity rows, live mask, parked rows not rendered   src/rtgs/image2gs/pool.py:55-120
  - park / activate: live mask + zeroed Adam moments of the rows     src/rtgs/image2gs/pool.py:123-151
  - residual spawn: top-k |target - render| pixels, isotropic seeds  src/rtgs/image2gs/pool.py:154-182
  - triage: park lowest weights (keep min live), spawn into free rows  src/rtgs/image2gs/pool.py:185-207
  - loop: render live rows, loss, step, sched, triage, PSNR log      src/rtgs/image2gs/pool.py:210-291
The renderer is ``oracle.render2d``; the loss is the reference's MSE (fit.py:557-563, no mask).
"""

from __future__ import annotations

import torch

from oracle import render2d
from oracle.fit import MIN_DIAG, build, psnr, to_raw

NAMES = ("xy_raw", "diag_raw", "off_raw", "color_raw", "weight_raw")


def _spawn(target, rendered, count):
    """(xy, chol, color, weight) of up to ``count`` seeds at the largest residuals (pool.py:154-182)."""
    height, width = target.shape[:2]
    flat = (target - rendered).abs().sum(dim=-1).reshape(-1)
    count = min(count, int((flat > 0).sum()))
    if count <= 0:
        return None
    idx = torch.topk(flat, count).indices
    py = (idx // width).to(target.dtype) + 0.5
    px = (idx % width).to(target.dtype) + 0.5
    scale = max((height * width / max(flat.numel(), 1)) ** 0.5 * 0.6, MIN_DIAG + 0.1)
    chol = torch.zeros(count, 3, dtype=target.dtype)
    chol[:, 0] = scale
    chol[:, 2] = scale
    color = target.reshape(-1, 3)[idx].clamp(1e-3, 1 - 1e-3)
    return torch.stack([px, py], dim=-1), chol, color, torch.full((count,), 0.5, dtype=target.dtype)


def fit_pooled(target, init, capacity, iterations, lr=1e-2, log_every=50, triage_every=50,
               prune_count=32, spawn_count=32, min_live=1):
    """Pooled fit of an (H, W, 3) target from (xy, chol, color, weight) of n <= capacity rows.

    Returns ((xy, chol, color, weight) of the live rows, history with psnr / final_psnr / live_count).
    """
    height, width = target.shape[:2]
    xy0, chol0, color0, weight0 = init
    n = xy0.shape[0]
    seed = to_raw(xy0, chol0, color0, weight0, height, width)
    raw = {}
    for name in NAMES:
        buf = torch.zeros((capacity, *seed[name].shape[1:]), dtype=target.dtype)
        buf[:n] = seed[name].detach()
        raw[name] = buf.requires_grad_(True)
    active = torch.zeros(capacity, dtype=torch.bool)
    active[:n] = True
    opt = torch.optim.Adam([raw[k] for k in NAMES], lr=lr)
    sched = torch.optim.lr_scheduler.CosineAnnealingLR(opt, T_max=iterations, eta_min=lr * 0.1)

    def render_live():
        rows = active.nonzero(as_tuple=True)[0]
        return render2d.render(*build({k: v[rows] for k, v in raw.items()}, height, width), height, width)

    def zero_moments(rows):
        for name in NAMES:
            state = opt.state.get(raw[name])
            if state:
                state["exp_avg"][rows] = 0.0
                state["exp_avg_sq"][rows] = 0.0

    hist = {"psnr": [], "stopped_iter": iterations - 1}
    for it in range(iterations):
        opt.zero_grad()
        rendered = render_live()
        torch.nn.functional.mse_loss(rendered, target).backward()
        opt.step()
        sched.step()
        if triage_every and (it + 1) % triage_every == 0 and it + 1 < iterations:
            live_count = int(active.sum())
            prune = min(prune_count, max(0, live_count - min_live))
            if prune > 0:
                live = active.nonzero(as_tuple=True)[0]
                with torch.no_grad():
                    weights = torch.sigmoid(raw["weight_raw"])[live]
                victims = live[torch.topk(weights, prune, largest=False).indices]
                active[victims] = False
                zero_moments(victims)
            free = (~active).nonzero(as_tuple=True)[0]
            budget = min(spawn_count, int(free.numel()))
            if budget > 0:
                with torch.no_grad():
                    seeds = _spawn(target, render_live(), budget)
                if seeds is not None:
                    rows = free[: seeds[0].shape[0]]
                    vals = to_raw(*seeds, height, width)
                    with torch.no_grad():
                        for name in NAMES:
                            raw[name].data[rows] = vals[name]
                    active[rows] = True
                    zero_moments(rows)
        if it % log_every == 0 or it == iterations - 1:
            with torch.no_grad():
                hist["psnr"].append((it, psnr(rendered.clamp(0, 1), target)))
    with torch.no_grad():
        rows = active.nonzero(as_tuple=True)[0]
        params = build({k: v[rows] for k, v in raw.items()}, height, width)
        final = render2d.render(*params, height, width)
    hist["final_psnr"] = psnr(final.clamp(0, 1), target)
    hist["live_count"] = int(rows.numel())
    return tuple(p.detach() for p in params), hist
