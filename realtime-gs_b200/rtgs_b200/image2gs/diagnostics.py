"""Native fit diagnostics: per-event snapshots of a fit (reference: src/rtgs/image2gs/fit.py:96-131
for the snapshot type, fit.py:423-520 for the events, fit.py:679-766 for their contents).

With a ``diagnostic_callback`` the fit advances one iteration at a time through the engine and
emits, like the reference's loop:

  ``initial``      step 0: the raw state, the initial render and its loss (no gradients yet);
  ``pre_update``   step k (k updates done): the gradients of the k-th loss as the engine's Adam
                   step receives them (``rtgs2d_fit_gradients``), the render and the loss;
  ``post_update``  step k + 1: the state after the update (gradients still those of step k);
  ``checkpoint``   step k + 1 when requested in ``diagnostic_steps``: a fresh render and loss.

Raw parameters, gradients and Adam moments come from the engine (the state the fit really
has); the optimizer's param groups, defaults and scheduler state come from a torch Adam +
CosineAnnealingLR of the same configuration stepped in lockstep over placeholder tensors, so
their structure is the installed torch's own. This path exists for research runs: it synchronises
with the device several times per iteration.
"""

from __future__ import annotations

from collections.abc import Callable, Collection
from dataclasses import dataclass
from typing import Any

import numpy as np
import torch

from rtgs_b200.core.gaussians2d import Gaussians2D
from rtgs_b200.image2gs.engine import FitEngine, psnr_values


@dataclass(frozen=True)
class NativeFitDiagnostic:
    """Detached snapshot of one event in a native fit (same fields as the reference's)."""

    event: str
    step: int
    appearance_parameterization: str
    geometry_frozen: bool
    initial_gaussians: Gaussians2D | None
    initializer_rng_state_before: torch.Tensor | None
    initializer_rng_state_after: torch.Tensor | None
    raw_parameters: dict[str, torch.Tensor]
    gradients: dict[str, torch.Tensor | None]
    gaussians: Gaussians2D
    target: torch.Tensor
    rendered: torch.Tensor | None
    loss: torch.Tensor | None
    optimizer_param_names: tuple[str, ...]
    optimizer_state: dict[str, dict[str, Any]]
    optimizer_param_groups: tuple[dict[str, Any], ...]
    optimizer_defaults: dict[str, Any]
    scheduler_state: dict[str, Any]
    lr_used: float | None
    next_lr: float


NativeFitDiagnosticCallback = Callable[[NativeFitDiagnostic], None]


def _clone(value: Any) -> Any:
    if isinstance(value, torch.Tensor):
        return value.detach().clone()
    if isinstance(value, dict):
        return {k: _clone(v) for k, v in value.items()}
    if isinstance(value, (list, tuple)):
        return type(value)(_clone(v) for v in value)
    return value


def fit_loss(rendered: torch.Tensor, target: torch.Tensor, mask: torch.Tensor | None) -> torch.Tensor:
    """The fit's data loss (fit.py:555-561): MSE, or the 0.1 + 0.9 mask weighted squared error."""
    if mask is None:
        return torch.nn.functional.mse_loss(rendered, target)
    weights = 0.1 + 0.9 * mask.to(rendered).clamp(0, 1)
    return (((rendered - target) ** 2) * weights[..., None]).mean()


class _ScheduleMirror:
    """torch Adam + CosineAnnealingLR(T_max=iterations, eta_min=0.1 lr) over one placeholder per
    optimised raw parameter, stepped once per fit iteration (no gradients, so no Adam state): the
    reference's optimizer bookkeeping, whose learning rates the engine's own recursion equals."""

    def __init__(self, names: tuple[str, ...], lr: float, iterations: int) -> None:
        self.names = names
        self.params = [torch.zeros(1, requires_grad=True) for _ in names]
        self.opt = torch.optim.Adam(self.params, lr=lr)
        self.sched = torch.optim.lr_scheduler.CosineAnnealingLR(self.opt, T_max=iterations, eta_min=lr * 0.1)

    @property
    def lr(self) -> float:
        return float(self.opt.param_groups[0]["lr"])

    def step(self) -> None:
        self.opt.step()
        self.sched.step()

    def param_groups(self) -> tuple[dict[str, Any], ...]:
        by_id = {id(p): n for p, n in zip(self.params, self.names)}
        return tuple({k: (tuple(by_id[id(p)] for p in v) if k == "params" else _clone(v)) for k, v in g.items()}
                     for g in self.opt.param_groups)


class DiagnosticFit:
    """Drives a one-view engine iteration by iteration and emits the reference's events."""

    def __init__(self, engine: FitEngine, *, config, g0: Gaussians2D, target: torch.Tensor,
                 mask: torch.Tensor | None, callback: NativeFitDiagnosticCallback, steps: Collection[int],
                 rng_state_before: torch.Tensor | None, rng_state_after: torch.Tensor | None,
                 coverage_fn=None) -> None:
        self.engine, self.config, self.g0, self.target, self.mask = engine, config, g0, target, mask
        self.callback = callback
        self.requested = frozenset(int(s) for s in steps)
        self.rng = (rng_state_before, rng_state_after)
        self.coverage_fn = coverage_fn
        names = tuple(name for name, _ in engine._raw_shapes)
        geometry = ("xy_raw", "diag_raw", "off_raw")
        self.raw_names = names
        self.opt_names = tuple(n for n in names if n not in geometry) if config.freeze_geometry else names
        self.mirror = _ScheduleMirror(self.opt_names, config.lr, config.iterations)
        self.updates = 0

    # -- engine state ----------------------------------------------------------------------------
    def _raw(self) -> dict[str, torch.Tensor]:
        return {k: v[0] for k, v in self.engine.raw().items()}

    def _built(self) -> Gaussians2D:
        xy, chol, color, weight = (t[0] for t in self.engine.params())
        return Gaussians2D(xy=xy, chol=chol, color=color, weight=weight)

    def _optimizer_state(self) -> dict[str, dict[str, Any]]:
        if self.updates == 0:
            return {n: {} for n in self.opt_names}
        m1, m2 = self.engine.moments()
        step = torch.tensor(float(self.updates))
        return {n: {"step": step.clone(), "exp_avg": m1[n][0], "exp_avg_sq": m2[n][0]} for n in self.opt_names}

    def _loss(self, rendered: torch.Tensor, built: Gaussians2D | None) -> torch.Tensor:
        loss = fit_loss(rendered, self.target, self.mask)
        if built is not None and self.coverage_fn is not None:
            loss = loss + self.coverage_fn(built)
        return loss

    def _emit(self, event: str, step: int, *, grads: dict[str, torch.Tensor] | None, built: Gaussians2D,
              rendered: torch.Tensor | None, loss: torch.Tensor | None, lr_used: float | None) -> None:
        initial = event == "initial"
        snap = NativeFitDiagnostic(
            event=event,
            step=step,
            appearance_parameterization=self.config.appearance_parameterization,
            geometry_frozen=self.config.freeze_geometry,
            initial_gaussians=self.g0.detach() if initial else None,
            initializer_rng_state_before=_clone(self.rng[0]) if initial else None,
            initializer_rng_state_after=_clone(self.rng[1]) if initial else None,
            raw_parameters=self._raw(),
            gradients={n: (None if grads is None or n not in self.opt_names else grads[n][0].clone())
                       for n in self.raw_names},
            gaussians=built.detach(),
            target=self.target.detach().clone(),
            rendered=None if rendered is None else rendered.detach().clone(),
            loss=None if loss is None else loss.detach().clone(),
            optimizer_param_names=self.opt_names,
            optimizer_state=self._optimizer_state(),
            optimizer_param_groups=self.mirror.param_groups(),
            optimizer_defaults=_clone(self.mirror.opt.defaults),
            scheduler_state=_clone(self.mirror.sched.state_dict()),
            lr_used=lr_used,
            next_lr=self.mirror.lr,
        )
        rng_state = torch.random.get_rng_state()
        grad_enabled = torch.is_grad_enabled()
        try:
            self.callback(snap)
        finally:
            torch.random.set_rng_state(rng_state)
            torch.set_grad_enabled(grad_enabled)

    def _render(self) -> torch.Tensor:
        render, _ = self.engine.evaluate(want_render=True)
        return render[0]

    # -- the loop --------------------------------------------------------------------------------
    def run(self, counts: np.ndarray, patience: int, check_every: int, tol: float) -> int:
        """Run the fit; returns the iteration it stopped at (early stopping as the plain loop)."""
        iterations = self.config.iterations
        built = self._built()
        render = self._render()
        self._emit("initial", 0, grads=None, built=built, rendered=render, loss=self._loss(render, None),
                   lr_used=None)
        best, stale = -float("inf"), 0
        for it in range(iterations):
            grads, rendered, _ = self.engine.gradients(want_render=True)
            rendered = rendered[0]
            lr_used = self.mirror.lr
            self._emit("pre_update", it, grads=grads, built=built, rendered=rendered,
                       loss=self._loss(rendered, built), lr_used=lr_used)
            self.engine.run(1)
            self.updates += 1
            self.mirror.step()
            built = self._built()
            self._emit("post_update", it + 1, grads=grads, built=built, rendered=None, loss=None, lr_used=lr_used)
            if it + 1 in self.requested:
                render = self._render()
                self._emit("checkpoint", it + 1, grads=grads, built=built, rendered=render,
                           loss=self._loss(render, None), lr_used=lr_used)
            if patience and (it + 1) % check_every == 0:
                _, sums = self.engine.history()
                cur = psnr_values(sums[-1, :, 1], counts)[0]
                if cur > best + tol:
                    best, stale = cur, 0
                else:
                    stale += 1
                    if stale >= patience:
                        return it
        return iterations - 1
