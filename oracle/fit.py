"""CPU oracle: the native Stage-1 fit loop, restated from the reference.

TEST INFRASTRUCTURE ONLY -- imported by tests/, __graft_entry__.smoke() and bench.py's CPU
baseline leg; never by the product package.

Restated reference behaviour (paths relative to the reference project):
  - raw reparameterisation and its inverse   src/rtgs/image2gs/fit.py:374-417
    (both appearance parameterisations: weight_color_9p and unit_weight_bounded_8p, whose
    amplitude_raw = logit(sigmoid(weight_raw) * sigmoid(color_raw)) and weight = 1)
  - torch Adam + CosineAnnealingLR(eta_min=0.1*lr)   src/rtgs/image2gs/fit.py:419-422
  - loop: zero_grad, build, render, MSE, backward, step, sched, PSNR log   fit.py:451-540
  - final render and PSNR                    src/rtgs/image2gs/fit.py:542-554
  - stacked multi-view loop, loss = sum_b mean_b   src/rtgs/image2gs/batched.py:79-170
  - serial masked loss + mask coverage penalty  src/rtgs/image2gs/fit.py:457-459,557-572
  - psnr                                     src/rtgs/core/metrics.py:12-15
The renderer is ``oracle.render2d`` (the reference's pure-PyTorch scatter renderer, restated).
A mask-restricted loss (mean over mask pixels x 3 channels, the denominator of
``masked_psnr`` in src/rtgs/core/metrics.py:18-29) is provided for the masked batched workload,
which the reference's batched path does not implement (batched.py:55-56 rejects masks).
"""

from __future__ import annotations

import torch

from oracle import render2d

MIN_DIAG = 0.3
WEIGHT_COLOR_9P = "weight_color_9p"
UNIT_WEIGHT_8P = "unit_weight_bounded_8p"


def softplus_inv(x: torch.Tensor) -> torch.Tensor:
    return x + torch.log(-torch.expm1(-x))


def to_raw(xy, chol, color, weight, height: int, width: int,
           appearance: str = WEIGHT_COLOR_9P) -> dict[str, torch.Tensor]:
    """Raw (unconstrained) parameters from constrained ones (fit.py:375-387); works on (..., k)."""
    wh = xy.new_tensor([width, height])
    color_raw = torch.logit(color.clamp(1e-3, 1 - 1e-3))
    weight_raw = torch.logit(weight.clamp(1e-3, 1 - 1e-3))
    raw = {
        "xy_raw": torch.logit((xy / wh).clamp(1e-4, 1 - 1e-4)),
        "diag_raw": softplus_inv(chol[..., [0, 2]] - MIN_DIAG),
        "off_raw": chol[..., 1].clone(),
    }
    if appearance == WEIGHT_COLOR_9P:
        raw.update(color_raw=color_raw, weight_raw=weight_raw)
    elif appearance == UNIT_WEIGHT_8P:
        raw["amplitude_raw"] = torch.logit(torch.sigmoid(weight_raw)[..., None] * torch.sigmoid(color_raw))
    else:
        raise ValueError(f"unknown appearance parameterisation {appearance!r}")
    return raw


def appearance_names(raw: dict[str, torch.Tensor]) -> tuple[str, ...]:
    """The raw parameters a geometry-frozen fit optimises (fit.py:393-397)."""
    return ("amplitude_raw",) if "amplitude_raw" in raw else ("color_raw", "weight_raw")


def build(raw: dict[str, torch.Tensor], height: int, width: int):
    """Constrained (xy, chol, color, weight) from raw parameters (fit.py:402-417)."""
    wh = raw["xy_raw"].new_tensor([width, height])
    diag = torch.nn.functional.softplus(raw["diag_raw"]) + MIN_DIAG
    chol = torch.stack([diag[..., 0], raw["off_raw"], diag[..., 1]], dim=-1)
    if "amplitude_raw" in raw:
        color = torch.sigmoid(raw["amplitude_raw"])
        weight = torch.ones_like(color[..., 0])
    else:
        color = torch.sigmoid(raw["color_raw"])
        weight = torch.sigmoid(raw["weight_raw"])
    return torch.sigmoid(raw["xy_raw"]) * wh, chol, color, weight


def psnr(pred: torch.Tensor, target: torch.Tensor) -> float:
    mse = torch.nn.functional.mse_loss(pred, target).clamp_min(1e-12)
    return float(-10.0 * torch.log10(mse))


def masked_psnr(pred: torch.Tensor, target: torch.Tensor, mask: torch.Tensor) -> float:
    w = mask.to(pred).clamp(0, 1)
    mse = (((pred - target) ** 2) * w[..., None]).sum() / (w.sum() * pred.shape[-1])
    return float(-10.0 * torch.log10(mse.clamp_min(1e-12)))


class StackedFit:
    """The stacked-view fit loop, one iteration per ``step`` (``fit_views`` runs it to the end;
    bench.py's CPU baseline times single iterations of it from any parameter state)."""

    def __init__(self, targets, init, iterations, lr=1e-2, masks=None, freeze_geometry=False, t_max=None,
                 appearance=WEIGHT_COLOR_9P, budget=render2d.DEFAULT_BUDGET):
        self.targets, self.masks = targets, masks
        self.budget = budget  # pairs per index_add chunk (the time; gradients only to float32 rounding)
        self.n_views, self.height, self.width = targets.shape[:3]
        self.raw = to_raw(*init, self.height, self.width, appearance)
        names = appearance_names(self.raw) if freeze_geometry else tuple(self.raw)
        for name, value in self.raw.items():
            value.requires_grad_(name in names)
        self.opt = torch.optim.Adam([self.raw[n] for n in names], lr=lr)
        self.sched = torch.optim.lr_scheduler.CosineAnnealingLR(self.opt, T_max=t_max or iterations,
                                                                eta_min=lr * 0.1)
        self.hist = [{"psnr": [], "stopped_iter": iterations - 1} for _ in range(self.n_views)]
        if masks is not None:
            self.mw = masks.to(targets).clamp(0, 1)
            self.denom = self.mw.sum(dim=(1, 2)) * 3.0

    def _psnr(self, pred, b):
        if self.masks is None:
            return psnr(pred, self.targets[b])
        return masked_psnr(pred, self.targets[b], self.masks[b])

    def step(self, it: int, log: bool = False) -> None:
        self.opt.zero_grad()
        xy, chol, color, weight = build(self.raw, self.height, self.width)
        rendered = render2d.render_batched(xy, chol, color, weight, self.height, self.width, budget=self.budget)
        if self.masks is None:
            loss = (rendered - self.targets).square().mean(dim=(1, 2, 3)).sum()
        else:
            loss = (((rendered - self.targets) ** 2) * self.mw[..., None]).sum(dim=(1, 2, 3)).div(self.denom).sum()
        if log:
            with torch.no_grad():
                for b in range(self.n_views):
                    self.hist[b]["psnr"].append((it, self._psnr(rendered[b].clamp(0, 1), b)))
        loss.backward()
        self.opt.step()
        self.sched.step()

    def finish(self):
        with torch.no_grad():
            xy, chol, color, weight = build(self.raw, self.height, self.width)
            final = render2d.render_batched(xy, chol, color, weight, self.height, self.width, budget=self.budget)
            for b in range(self.n_views):
                pred = final[b].clamp(0, 1)
                self.hist[b]["final_psnr_full"] = psnr(pred, self.targets[b])
                self.hist[b]["final_psnr"] = self._psnr(pred, b)
        return (xy, chol, color, weight), self.hist


def fit_views(
    targets: torch.Tensor,
    init: tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor],
    iterations: int,
    lr: float = 1e-2,
    log_every: int = 50,
    masks: torch.Tensor | None = None,
    freeze_geometry: bool = False,
    t_max: int | None = None,
    appearance: str = WEIGHT_COLOR_9P,
    budget: int = render2d.DEFAULT_BUDGET,
):
    """Fit stacked (B, H, W, 3) targets from a stacked (B, N, .) initialisation.

    Returns (params (xy, chol, color, weight) stacked, histories). With B == 1 and no mask this is
    the single-image native fit (the per-view MSE mean is the serial loss); with a (B, H, W) mask
    the loss is the mask-restricted mean and PSNR is ``masked_psnr``. ``t_max`` (default
    ``iterations``) is the cosine schedule's length, so the first iterations of a longer fit can be
    run alone. ``appearance`` selects the raw appearance parameters (fit.py:381-387). ``budget`` is
    the pairs per index_add chunk (``render2d.reference_budget`` for the reference's).
    """
    fit = StackedFit(targets, init, iterations, lr=lr, masks=masks, freeze_geometry=freeze_geometry, t_max=t_max,
                     appearance=appearance, budget=budget)
    for it in range(iterations):
        fit.step(it, log=it % log_every == 0 or it == iterations - 1)
    return fit.finish()


def fit_serial(target, init, iterations, lr=1e-2, log_every=50, mask=None, coverage_weight=0.0,
               appearance=WEIGHT_COLOR_9P, image=None):
    """The serial native fit loop (fit.py:451-554) of one (H, W, 3) target, with the serial loss
    (fit.py:557-563: MSE, or (0.1 + 0.9 mask)-weighted MSE with a mask) and the optional mask
    coverage penalty weight * mean(coverage * (1 - mask)), coverage = 1 - exp(-density)
    (fit.py:457-459, 566-572; renderer2d.py:128-140). Returns ((xy, chol, color, weight), history).

    With a mask, the reference fits the masked image (target = image * mask, fit.py:333-336) and
    reports final_psnr = masked_psnr of the final render against the unmasked ``image``
    (fit.py:546-552; ``image`` defaults to ``target``), final_psnr_full = PSNR against the target.
    """
    height, width = target.shape[:2]
    raw = to_raw(*init, height, width, appearance)
    for value in raw.values():
        value.requires_grad_(True)
    opt = torch.optim.Adam(list(raw.values()), lr=lr)
    sched = torch.optim.lr_scheduler.CosineAnnealingLR(opt, T_max=iterations, eta_min=lr * 0.1)
    hist = {"psnr": [], "stopped_iter": iterations - 1}
    for it in range(iterations):
        opt.zero_grad()
        xy, chol, color, weight = build(raw, height, width)
        rendered, density = render2d.render_batched(xy[None], chol[None], color[None], weight[None],
                                                    height, width, with_density=True)
        rendered, density = rendered[0], density[0]
        if mask is None:
            loss = torch.nn.functional.mse_loss(rendered, target)
        else:
            wts = 0.1 + 0.9 * mask.to(rendered).clamp(0, 1)
            loss = (((rendered - target) ** 2) * wts[..., None]).mean()
            if coverage_weight > 0.0:
                coverage = 1.0 - torch.exp(-density)
                loss = loss + coverage_weight * (coverage * (1.0 - mask.to(coverage).clamp(0, 1))).mean()
        loss.backward()
        opt.step()
        sched.step()
        if it % log_every == 0 or it == iterations - 1:
            with torch.no_grad():
                hist["psnr"].append((it, psnr(rendered.clamp(0, 1), target)))
    with torch.no_grad():
        params = build(raw, height, width)
        final = render2d.render(*params, height, width)
    hist["final_psnr_full"] = psnr(final.clamp(0, 1), target)
    hist["final_psnr"] = hist["final_psnr_full"] if mask is None else masked_psnr(
        final.clamp(0, 1), target if image is None else image, mask)
    return tuple(p.detach() for p in params), hist


def adam_first_step(raw: torch.Tensor, grad: torch.Tensor, lr: float) -> torch.Tensor:
    """Closed form of torch Adam's first update (bias-corrected; betas 0.9/0.999, eps 1e-8).

    Mirrors the reference's own pin of the first update (tests/test_stage1_fit_seam.py:239-254).
    """
    beta1, beta2, eps = 0.9, 0.999, 1e-8
    exp_avg = (1 - beta1) * grad
    exp_avg_sq = (1 - beta2) * grad * grad
    step_size = lr / (1.0 - beta1)
    denom = exp_avg_sq.sqrt() / (1.0 - beta2) ** 0.5 + eps
    return raw - step_size * exp_avg / denom
