"""Pooled (fixed-capacity, free-list) Stage-1 fitting (reference: src/rtgs/image2gs/pool.py).

``FitConfig.pool`` fits with ``capacity`` parameter rows allocated once. A byte/bool live mask
selects the rows that are rendered; the others are spares. The renderer is additive (a pixel is the
plain sum of its gaussians' weighted colours), so leaving a row out of the render removes exactly
its contribution and gives it an exactly zero gradient: parking and reviving rows needs no tensor
resize and no new optimizer, only row writes and a reset of the touched rows' optimizer moments.

What lives here:
* ``fit_pooled_from_initialization`` (reference pool.py:210-291) runs the pooled fit inside the
  native fit engine. The live mask is the engine's own (``rtgs2d_fit_set_active``: its projection
  gives parked rows no tile entries), and rows are revived with ``rtgs2d_fit_write_rows`` (new raw
  values plus zeroed Adam moments, in place on the device). Between engine runs a triage event
  parks the weakest live rows and spawns new rows at the largest residuals of the engine's own
  render of the current state.
* ``GaussianPool2D`` (reference pool.py:55-151) is the same row lifecycle for callers that render
  with ``render_gaussians_2d`` and step their own torch optimizer: five raw leaf tensors of
  ``capacity`` rows in the optimizer's parameter order, the live mask, and park / activate, which
  reset every per-row state tensor the optimizer keeps for the touched rows.
"""

from __future__ import annotations

from typing import TYPE_CHECKING

import numpy as np
import torch

from rtgs_b200 import _native
from rtgs_b200.core.gaussians2d import Gaussians2D
from rtgs_b200.core.metrics import masked_psnr, psnr
from rtgs_b200.image2gs.engine import acquire_engine, pack_mask_bits, psnr_values, release_engine
from rtgs_b200.image2gs.fit import (
    _MIN_DIAG,
    _history_from_engine,
    _validate_initial_gaussians,
    raw_from_gaussians,
)

if TYPE_CHECKING:
    from rtgs_b200.image2gs.fit import FitConfig

# The raw fields of one row, in the order an optimizer receives them (the engine's order too).
RAW_FIELDS = ("xy_raw", "diag_raw", "off_raw", "color_raw", "weight_raw")

# Spawned rows start isotropic with this Cholesky diagonal: the reference sizes them as
# 0.6 * sqrt(H * W / (number of residual pixels)), floored at _MIN_DIAG + 0.1, and the residual
# map always has H * W pixels (pool.py:170), so the size is 0.6 pixels at every image size.
SPAWN_DIAG = 0.6
SPAWN_WEIGHT = 0.5


def _raw_rows(g: Gaussians2D, wh: torch.Tensor) -> dict[str, torch.Tensor]:
    """Raw rows of ``g`` for an image of size wh = (W, H) (the fit's inverse transforms)."""
    return raw_from_gaussians(g.xy, g.chol, g.color, g.weight, float(wh[1]), float(wh[0]))


def _constrained(fields: dict[str, torch.Tensor], wh: torch.Tensor) -> Gaussians2D:
    """The fit's parameter transforms (fit.py:402-417) applied to raw rows; differentiable."""
    diag = torch.nn.functional.softplus(fields["diag_raw"]) + _MIN_DIAG
    return Gaussians2D(
        xy=torch.sigmoid(fields["xy_raw"]) * wh,
        chol=torch.stack([diag[:, 0], fields["off_raw"], diag[:, 1]], dim=-1),
        color=torch.sigmoid(fields["color_raw"]),
        weight=torch.sigmoid(fields["weight_raw"]),
    )


def _zero_optimizer_rows(optimizer: torch.optim.Optimizer, params: list[torch.Tensor], rows: torch.Tensor) -> None:
    """Zero, at ``rows``, every state tensor the optimizer keeps per parameter row (Adam's two
    moments; any optimizer whose state tensors have the parameter's shape)."""
    for param in params:
        for value in optimizer.state.get(param, {}).values():
            if isinstance(value, torch.Tensor) and value.shape == param.shape:
                value[rows] = 0.0


class GaussianPool2D:
    """``capacity`` raw parameter rows with a live mask (API of the reference's pool.py:55-151).

    Rows ``[0, g0.n)`` start live with ``g0``'s parameters, the rest are parked spares. ``params()``
    are the five raw leaf tensors to hand to an optimizer; they are never reallocated.
    """

    def __init__(self, g0: Gaussians2D, wh: torch.Tensor, capacity: int):
        if capacity < g0.n:
            raise ValueError(f"pool capacity {capacity} is below the initial count {g0.n}")
        self.capacity = int(capacity)
        self.wh = wh
        seed = _raw_rows(g0, wh)
        self._leaves: dict[str, torch.Tensor] = {}
        for name in RAW_FIELDS:
            rows = seed[name].detach()
            leaf = rows.new_zeros((self.capacity, *rows.shape[1:]))
            leaf[: g0.n] = rows
            self._leaves[name] = leaf.requires_grad_(True)
        self.active = torch.arange(self.capacity, device=g0.xy.device) < g0.n

    def params(self) -> list[torch.Tensor]:
        """The raw leaf tensors, in optimizer order."""
        return [self._leaves[name] for name in RAW_FIELDS]

    @property
    def live_count(self) -> int:
        return int(self.active.sum())

    def active_indices(self) -> torch.Tensor:
        return torch.nonzero(self.active).flatten()

    def free_rows(self) -> torch.Tensor:
        """Parked rows in ascending order: the order in which spawns take them."""
        return torch.nonzero(~self.active).flatten()

    def _build_rows(self, rows: torch.Tensor) -> Gaussians2D:
        return _constrained({name: leaf[rows] for name, leaf in self._leaves.items()}, self.wh)

    def build_active(self) -> Gaussians2D:
        """The live rows as differentiable gaussians; parked rows are simply absent."""
        return self._build_rows(self.active_indices())

    def to_gaussians2d(self) -> Gaussians2D:
        """Detached copy of the live rows."""
        with torch.no_grad():
            return self._build_rows(self.active_indices()).detach()

    def built_weights(self) -> torch.Tensor:
        """Amplitudes of all ``capacity`` rows (parked rows report their stored value), detached."""
        with torch.no_grad():
            return torch.sigmoid(self._leaves["weight_raw"])

    def park(self, rows: torch.Tensor, optimizer: torch.optim.Optimizer) -> None:
        """Stop rendering ``rows`` and clear their optimizer state."""
        self.active[rows] = False
        _zero_optimizer_rows(optimizer, self.params(), rows)

    def activate(self, rows: torch.Tensor, gaussians: Gaussians2D, optimizer: torch.optim.Optimizer) -> None:
        """Overwrite ``rows`` with ``gaussians`` (in place), render them again, clear their state."""
        new = _raw_rows(gaussians, self.wh)
        with torch.no_grad():
            for name, leaf in self._leaves.items():
                leaf[rows] = new[name].to(leaf)
        self.active[rows] = True
        _zero_optimizer_rows(optimizer, self.params(), rows)


def _spawn_raw(target: torch.Tensor, rendered: torch.Tensor, mask: torch.Tensor | None, count: int,
               wh: torch.Tensor) -> dict[str, torch.Tensor] | None:
    """Raw rows of up to ``count`` new gaussians at the pixels of largest residual (reference
    pool.py:154-182): residual = |target - render| summed over the channels (times the mask),
    the ``count`` largest by torch.topk (ties in topk's order), only pixels with a non-zero
    residual. Each sits at its pixel centre, isotropic with diagonal SPAWN_DIAG, with the target's
    colour (clamped to [1e-3, 1 - 1e-3]) and weight SPAWN_WEIGHT."""
    width = target.shape[1]
    residual = (target - rendered).abs().sum(dim=-1)
    if mask is not None:
        residual = residual * mask.to(residual).clamp(0, 1)
    residual = residual.reshape(-1)
    count = min(count, int(torch.count_nonzero(residual)))
    if count <= 0:
        return None
    pick = torch.topk(residual, count).indices
    centre = torch.stack([pick % width, pick // width], dim=-1).to(target.dtype) + 0.5
    chol = centre.new_zeros(count, 3)
    chol[:, 0::2] = SPAWN_DIAG
    seeds = Gaussians2D(xy=centre, chol=chol,
                        color=target.reshape(-1, 3)[pick].clamp(1e-3, 1 - 1e-3),
                        weight=centre.new_full((count,), SPAWN_WEIGHT))
    return _raw_rows(seeds, wh)


def _triage(engine, active: torch.Tensor, target: torch.Tensor, mask: torch.Tensor | None,
            config: FitConfig, wh: torch.Tensor) -> None:
    """One triage event on the engine's rows (reference pool.py:185-207): park the lowest-amplitude
    live rows (keeping at least ``pool_min_live``), then spawn into the lowest free rows at the
    residual peaks of the engine's render of the remaining live set."""
    live = torch.nonzero(active).flatten()
    n_park = min(config.pool_prune_count, max(0, live.numel() - config.pool_min_live))
    if n_park > 0:
        amplitude = torch.sigmoid(engine.raw()["weight_raw"][0, live])
        parked = live[torch.topk(amplitude, n_park, largest=False).indices]
        active[parked] = False
        engine.write_rows(parked)  # zero their moments; the values stay (parked rows are inert)
    free = torch.nonzero(~active).flatten()
    engine.set_active(active[None])
    budget = min(config.pool_spawn_count, free.numel())
    if budget <= 0:
        return
    render, _ = engine.evaluate(want_render=True)
    seeds = _spawn_raw(target, render[0], mask, budget, wh)
    if seeds is None:
        return
    rows = free[: seeds["weight_raw"].shape[0]]
    engine.write_rows(rows, seeds)
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
        final, sums = engine.evaluate(want_render=mask is not None)
        ok = True
    finally:
        engine.set_active(None)
        release_engine(engine, reusable=ok)
    live = active.nonzero(as_tuple=True)[0]
    result = Gaussians2D(xy=xy[live], chol=chol[live], color=color[live], weight=weight[live])
    if mask is None:  # as the native fit: from the evaluation's clamped squared-error sum
        history["final_psnr_full"] = psnr_values(sums[:, 1], counts)[0]
        history["final_psnr"] = history["final_psnr_full"]
    else:
        pred = final[0].clamp(0, 1)
        history["final_psnr_full"] = psnr(pred, target)
        history["final_psnr"] = masked_psnr(pred, image, mask)
    history["live_count"] = int(live.numel())
    history["pool_capacity"] = capacity
    result.xy += xy_offset
    return result, history
