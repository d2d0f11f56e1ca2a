"""Fixed-capacity 2D-gaussian pool with a free list (reference: rtgs/image2gs/pool.py).

Opt-in (``FitConfig.pool``). ``capacity`` raw-parameter rows exist for the whole fit; a boolean
``active`` mask marks live rows and the parked rows form the free list. The compositor is additive,
so a parked row is simply not rendered: its contribution and its gradient are exactly zero. Periodic
triage parks the lowest-weight live rows and spawns new rows at the pixels of largest residual,
writing parameters in place and zeroing only the touched rows' Adam moments.

Two layers, as in the reference:
* ``GaussianPool2D`` -- the row store with torch-optimizer park/activate (pool.py:55-151), for
  callers that drive their own optimizer;
* ``fit_pooled_from_initialization`` (pool.py:210-291) -- the pooled fit, run by the native fit
  engine: parked rows are excluded by the engine's projection (``rtgs2d_fit_set_active``), and park
  / activate become in-place row writes with moment resets (``rtgs2d_fit_write_rows``); the triage
  itself runs between engine runs, on the device, with torch ops.
"""

from __future__ import annotations

from typing import TYPE_CHECKING

import numpy as np
import torch

from rtgs_b200.core.gaussians2d import Gaussians2D
from rtgs_b200 import _native
from rtgs_b200.core.metrics import masked_psnr, psnr
from rtgs_b200.image2gs.engine import acquire_engine, pack_mask_bits, psnr_values, release_engine
from rtgs_b200.image2gs.fit import (
    _MIN_DIAG,
    _history_from_engine,
    _softplus_inv,
    _validate_initial_gaussians,
    raw_from_gaussians,
)

if TYPE_CHECKING:
    from rtgs_b200.image2gs.fit import FitConfig

# Raw parameter names, in optimizer order (pool.py:41).
_RAW_NAMES = ("xy_raw", "diag_raw", "off_raw", "color_raw", "weight_raw")


def _raw_from_gaussians(g: Gaussians2D, wh: torch.Tensor) -> dict[str, torch.Tensor]:
    """Unconstrained parameters of ``g`` (pool.py:44-52)."""
    return {
        "xy_raw": torch.logit((g.xy / wh).clamp(1e-4, 1 - 1e-4)),
        "diag_raw": _softplus_inv(g.chol[:, [0, 2]] - _MIN_DIAG),
        "off_raw": g.chol[:, 1].clone(),
        "color_raw": torch.logit(g.color.clamp(1e-3, 1 - 1e-3)),
        "weight_raw": torch.logit(g.weight.clamp(1e-3, 1 - 1e-3)),
    }


class GaussianPool2D:
    """Fixed-capacity raw-parameter store with an ``active`` / free-list row lifecycle (pool.py:55-151)."""

    def __init__(self, g0: Gaussians2D, wh: torch.Tensor, capacity: int):
        if capacity < g0.n:
            raise ValueError(f"pool capacity {capacity} is below the initial count {g0.n}")
        device, dtype = g0.xy.device, g0.xy.dtype
        self.capacity = int(capacity)
        self.wh = wh
        self._raw: dict[str, torch.Tensor] = {}
        seed = _raw_from_gaussians(g0, wh)
        for name in _RAW_NAMES:
            init = seed[name]
            buffer = torch.zeros((capacity, *init.shape[1:]), device=device, dtype=dtype)
            buffer[: g0.n] = init.detach()
            buffer.requires_grad_(True)
            self._raw[name] = buffer
        self.active = torch.zeros(capacity, dtype=torch.bool, device=device)
        self.active[: g0.n] = True

    def params(self) -> list[torch.Tensor]:
        """The raw leaf tensors, in optimizer order."""
        return [self._raw[name] for name in _RAW_NAMES]

    @property
    def live_count(self) -> int:
        return int(self.active.sum())

    def active_indices(self) -> torch.Tensor:
        return self.active.nonzero(as_tuple=True)[0]

    def free_rows(self) -> torch.Tensor:
        """Parked-row indices (the free list), ascending -- the deterministic spend order."""
        return (~self.active).nonzero(as_tuple=True)[0]

    def _build_rows(self, rows: torch.Tensor) -> Gaussians2D:
        diag = torch.nn.functional.softplus(self._raw["diag_raw"][rows]) + _MIN_DIAG
        chol = torch.stack([diag[:, 0], self._raw["off_raw"][rows], diag[:, 1]], dim=-1)
        return Gaussians2D(
            xy=torch.sigmoid(self._raw["xy_raw"][rows]) * self.wh,
            chol=chol,
            color=torch.sigmoid(self._raw["color_raw"][rows]),
            weight=torch.sigmoid(self._raw["weight_raw"][rows]),
        )

    def build_active(self) -> Gaussians2D:
        """Differentiable live-only gaussians (parked rows are omitted -> zero contribution)."""
        return self._build_rows(self.active_indices())

    def to_gaussians2d(self) -> Gaussians2D:
        """Detached snapshot of the live rows."""
        with torch.no_grad():
            return self._build_rows(self.active_indices()).detach()

    def built_weights(self) -> torch.Tensor:
        """Detached ``(capacity,)`` amplitudes; parked rows report their stored (unused) value."""
        with torch.no_grad():
            return torch.sigmoid(self._raw["weight_raw"])

    def _zero_moments(self, optimizer: torch.optim.Optimizer, rows: torch.Tensor) -> None:
        for param in self.params():
            state = optimizer.state.get(param)
            if not state:
                continue
            for key in ("exp_avg", "exp_avg_sq"):
                if key in state:
                    state[key][rows] = 0.0

    def park(self, rows: torch.Tensor, optimizer: torch.optim.Optimizer) -> None:
        """Return ``rows`` to the free list; clears their optimizer momentum."""
        self.active[rows] = False
        self._zero_moments(optimizer, rows)

    def activate(self, rows: torch.Tensor, gaussians: Gaussians2D, optimizer: torch.optim.Optimizer) -> None:
        """Write ``gaussians`` into free ``rows`` in place, mark them live, reset their moments."""
        raw = _raw_from_gaussians(gaussians, self.wh)
        with torch.no_grad():
            for name in _RAW_NAMES:
                self._raw[name].data[rows] = raw[name].to(self._raw[name])
        self.active[rows] = True
        self._zero_moments(optimizer, rows)


def _residual_spawn_gaussians(
    target: torch.Tensor, rendered: torch.Tensor, mask: torch.Tensor | None, count: int
) -> Gaussians2D | None:
    """Seed up to ``count`` gaussians at the highest-error pixels, deterministic top-k (pool.py:154-182)."""
    height, width = target.shape[:2]
    error = (target - rendered).abs().sum(dim=-1)
    if mask is not None:
        error = error * mask.to(error).clamp(0, 1)
    flat = error.reshape(-1)
    count = min(count, int((flat > 0).sum()))
    if count <= 0:
        return None
    idx = torch.topk(flat, count).indices
    py = (idx // width).to(target.dtype) + 0.5
    px = (idx % width).to(target.dtype) + 0.5
    scale = max((height * width / max(flat.numel(), 1)) ** 0.5 * 0.6, _MIN_DIAG + 0.1)
    chol = torch.zeros(count, 3, device=target.device, dtype=target.dtype)
    chol[:, 0] = scale
    chol[:, 2] = scale
    return Gaussians2D(
        xy=torch.stack([px, py], dim=-1),
        chol=chol,
        color=target.reshape(-1, 3)[idx].clamp(1e-3, 1 - 1e-3),
        weight=torch.full((count,), 0.5, device=target.device, dtype=target.dtype),
    )


def _triage(engine, active: torch.Tensor, target: torch.Tensor, mask: torch.Tensor | None,
            config: FitConfig, wh: torch.Tensor) -> None:
    """One in-place triage event on the engine's rows (pool.py:185-207): park the lowest-amplitude
    live rows (keeping ``pool_min_live``), then spawn at the current residual peaks."""
    live_count = int(active.sum())
    prune = min(config.pool_prune_count, max(0, live_count - config.pool_min_live))
    if prune > 0:
        live = active.nonzero(as_tuple=True)[0]
        weights = torch.sigmoid(engine.raw()["weight_raw"][0])[live]
        victims = live[torch.topk(weights, prune, largest=False).indices]
        active[victims] = False
        engine.write_rows(victims)  # moments only
    free = (~active).nonzero(as_tuple=True)[0]
    budget = min(config.pool_spawn_count, int(free.numel()))
    engine.set_active(active[None])
    if budget > 0:
        rendered, _ = engine.evaluate(want_render=True)
        seeds = _residual_spawn_gaussians(target, rendered[0], mask, budget)
        if seeds is not None:
            rows = free[: seeds.n]
            engine.write_rows(rows, _raw_from_gaussians(seeds, wh))
            active[rows] = True
            engine.set_active(active[None])


def fit_pooled_from_initialization(
    image: torch.Tensor,
    target: torch.Tensor,
    g0: Gaussians2D,
    config: FitConfig,
    mask: torch.Tensor | None,
    xy_offset: torch.Tensor,
) -> tuple[Gaussians2D, dict]:
    """Pooled fit from a supplied initialisation (pool.py:210-291), on the native fit engine.

    Returns the live gaussians (ascending row order, restored to full-image coordinates) and the
    usual history plus ``live_count`` and ``pool_capacity``.
    """
    height, width = image.shape[:2]
    _validate_initial_gaussians(g0, height, width)
    wh = image.new_tensor([width, height])
    capacity = config.pool_capacity or config.max_gaussians or (2 * config.n_gaussians)
    if capacity < g0.n:
        raise ValueError(f"pool capacity {capacity} is below the initial count {g0.n}")
    seed = raw_from_gaussians(g0.xy, g0.chol, g0.color, g0.weight, height, width)
    raw = {}
    for name, value in seed.items():
        buf = torch.zeros((capacity, *value.shape[1:]), device=image.device, dtype=torch.float32)
        buf[: g0.n] = value
        raw[name] = buf[None]
    active = torch.zeros(capacity, dtype=torch.bool, device=image.device)
    active[: g0.n] = True
    patience = int(config.convergence_patience)
    check_every = int(config.convergence_check_every) if patience else 0
    triage_every = int(config.pool_triage_every)
    engine = acquire_engine(
        1, capacity, height, width, lr=config.lr, iterations=config.iterations,
        log_every=config.log_every, check_every=check_every,
        loss_mode=_native.LOSS_MSE if mask is None else _native.LOSS_MASK_WEIGHTED,
        device=image.device,
    )
    ok = False
    try:
        engine.set_targets(target[None], None if mask is None else pack_mask_bits(mask[None]))
        engine.set_raw(raw)
        engine.set_active(active[None])
        counts = np.array([3.0 * height * width])
        stopped = config.iterations - 1
        best, stale = -float("inf"), 0
        done = 0
        while done < config.iterations:
            # Run up to the next triage or convergence check (both act after an iteration's step).
            stop = config.iterations
            if triage_every:
                stop = min(stop, (done // triage_every + 1) * triage_every)
            if check_every:
                stop = min(stop, (done // check_every + 1) * check_every)
            engine.run(stop - done)
            done = stop
            if triage_every and done % triage_every == 0 and done < config.iterations:
                _triage(engine, active, target, mask, config, wh)
            if check_every and done % check_every == 0:
                _, sums = engine.history()
                cur = psnr_values(sums[-1, :, 1], counts)[0]
                if cur > best + config.convergence_tol:
                    best, stale = cur, 0
                else:
                    stale += 1
                    if stale >= patience:
                        stopped = done - 1
                        break
        history = _history_from_engine(engine, config, counts)[0]
        if stopped != config.iterations - 1:
            history["psnr"] = [(i, v) for i, v in history["psnr"] if i <= stopped]
            history["stopped_iter"] = stopped
        xy, chol, color, weight = (t[0] for t in engine.params())
        final, _ = engine.evaluate(want_render=True)
        ok = True
    finally:
        engine.set_active(None)
        release_engine(engine, reusable=ok)
    live = active.nonzero(as_tuple=True)[0]
    result = Gaussians2D(xy=xy[live], chol=chol[live], color=color[live], weight=weight[live])
    pred = final[0].clamp(0, 1)
    history["final_psnr_full"] = psnr(pred, target)
    history["final_psnr"] = history["final_psnr_full"] if mask is None else masked_psnr(pred, image, mask)
    history["live_count"] = int(live.numel())
    history["pool_capacity"] = capacity
    result.xy += xy_offset
    return result, history
