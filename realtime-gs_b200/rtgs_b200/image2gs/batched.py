"""Fused multi-view Stage-1 fitting (reference: src/rtgs/image2gs/batched.py:39-170).

All views are fitted jointly by one C fit engine: identical per-view initialisation (generator
seeded ``seed + i`` on the image's device), stacked (B, N, .) raw parameters, one batched render
per iteration and loss = sum over views of the per-view MSE, so each view's gradient is its
serial-fit gradient. Same validation and history keys as the reference.

``masks`` are accepted here (the reference rejects them, batched.py:55-56) when
``mask_loss="mask_only"`` is requested through ``fit_views_batched_masked``: the loss is then the
squared error over mask pixels divided by 3 x mask pixels per view, i.e. the denominator of
``masked_psnr`` (metrics.py:27-28).
"""

from __future__ import annotations

import numpy as np
import torch

from rtgs_b200 import _native
from rtgs_b200.core.gaussians2d import Gaussians2D
from rtgs_b200.core.metrics import masked_psnr, psnr
from rtgs_b200.image2gs.engine import acquire_engine, pack_mask_bits, psnr_values, release_engine
from rtgs_b200.image2gs.fit import (
    FitConfig,
    _history_from_engine,
    _require_cuda,
    _validate_fit_controls,
    _validate_initial_gaussians,
    _validate_raw_parameters,
    init_gaussians_2d,
    raw_from_gaussians,
)


def _check_views(images: list[torch.Tensor]) -> tuple[int, int]:
    height, width = images[0].shape[:2]
    for image in images:
        if image.shape != images[0].shape:
            raise ValueError("batch_views requires equally sized views")
    return height, width


def fit_views_batched(
    images: list[torch.Tensor],
    config: FitConfig | None = None,
    seed: int = 0,
    masks: list[torch.Tensor] | None = None,
) -> tuple[list[Gaussians2D], list[dict]]:
    """Fit every view jointly in one fused optimisation; API mirrors ``fit_views``."""
    config = config or FitConfig()
    _validate_fit_controls(config)
    if masks is not None and any(mask is not None for mask in masks):
        raise ValueError("batch_views does not support masks; use serial fit_views")
    if config.convergence_patience:
        raise ValueError("batch_views does not support convergence early stopping")
    if not images:
        return [], []
    height, width = _check_views(images)
    inits = []
    for i, image in enumerate(images):
        _require_cuda(image)
        generator = torch.Generator(device=image.device).manual_seed(seed + i)
        g0 = init_gaussians_2d(image, config.n_gaussians, config.grad_init_mix, generator)
        _validate_initial_gaussians(g0, height, width)
        inits.append(g0)
    init = tuple(torch.stack([getattr(g, f) for g in inits]) for f in ("xy", "chol", "color", "weight"))
    return fit_stacked(torch.stack(images), init, config)


def fit_stacked(
    targets: torch.Tensor,
    init: tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor],
    config: FitConfig,
    masks: torch.Tensor | None = None,
) -> tuple[list[Gaussians2D], list[dict]]:
    """Fit stacked (B, H, W, 3) CUDA targets from a stacked (B, N, .) initialisation.

    With ``masks`` (B, H, W) the loss is restricted to mask pixels (mean over mask pixels x 3)
    and PSNR is ``masked_psnr``.
    """
    _require_cuda(targets)
    n_views, height, width = targets.shape[:3]
    xy0, chol0, color0, weight0 = (t.to(targets.device, torch.float32) for t in init)
    loss_mode = _native.LOSS_MSE if masks is None else _native.LOSS_MASK_ONLY
    engine = acquire_engine(
        n_views, xy0.shape[1], height, width, lr=config.lr, iterations=config.iterations,
        log_every=config.log_every, freeze_geometry=config.freeze_geometry, loss_mode=loss_mode,
        device=targets.device, appearance=config.appearance_parameterization,
    )
    ok = False
    try:
        # Raw transform on the device; like the reference's batched fit, only non-finite raw
        # parameters are rejected here (the per-view initialisers were validated by the caller).
        status = engine.set_initial(xy0, chol0, color0, weight0)
        if status & _native.INIT_NONFINITE_RAW:
            ok = True
            _validate_raw_parameters(raw_from_gaussians(xy0, chol0, color0, weight0, height, width,
                                                        config.appearance_parameterization))
            raise RuntimeError("the engine found non-finite raw parameters that the host check does not")
        mask_bits = None if masks is None else pack_mask_bits(masks)
        engine.set_targets(targets, mask_bits)
        engine.run(config.iterations)
        if masks is None:
            counts = np.full(n_views, 3.0 * height * width)
        else:
            counts = 3.0 * (masks.reshape(n_views, -1) > 0.5).sum(dim=1).double().cpu().numpy()
        histories = _history_from_engine(engine, config, counts)
        xy, chol, color, weight = engine.params()
        final, _ = engine.evaluate(want_render=True)
        ok = True
    finally:
        release_engine(engine, reusable=ok)
    for b in range(n_views):
        pred = final[b].clamp(0, 1)
        if masks is None:
            histories[b]["final_psnr_full"] = psnr(pred, targets[b])
            histories[b]["final_psnr"] = histories[b]["final_psnr_full"]
        else:
            histories[b]["final_psnr_full"] = psnr(pred, targets[b])
            histories[b]["final_psnr"] = masked_psnr(pred, targets[b], (masks[b] > 0.5).to(pred))
    results = [Gaussians2D(xy=xy[b], chol=chol[b], color=color[b], weight=weight[b]).detach() for b in range(n_views)]
    return results, histories


def fit_views_batched_masked(
    images: list[torch.Tensor],
    masks: list[torch.Tensor],
    init: tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor],
    config: FitConfig,
) -> tuple[list[Gaussians2D], list[dict]]:
    """Joint fit of masked views with the mask-restricted L2 loss (no reference counterpart)."""
    _validate_fit_controls(config)
    if len(images) != len(masks):
        raise ValueError("one mask per view is required")
    height, width = _check_views(images)
    for m in masks:
        if m.shape != (height, width):
            raise ValueError("mask size does not match image")
    return fit_stacked(torch.stack(images), init, config, masks=torch.stack(masks))
