"""Fit 2D gaussians to an image (reference: src/rtgs/image2gs/fit.py).

Same configuration object, initialiser, entry points and history dictionary as the reference's
native backend; the optimisation loop itself runs in the C fit engine (``engine.FitEngine``):
projection from raw parameters, tile binning, one fused forward + L2-gradient + backward kernel
and one fused chain-rule + Adam kernel per iteration, with torch's CosineAnnealingLR recursion
evaluated on the host.

Supported: ``backend="native"``, ``init_strategy="gradient"``, both appearance
parameterisations (weight_color_9p and unit_weight_bounded_8p, fit.py:381-411), fixed iterations
or convergence early stopping, ``freeze_geometry``, binary masks (crop + 0.1/0.9-weighted loss,
fit.py:262-269,557-563), native fit diagnostics (``diagnostic_callback`` / ``diagnostic_steps``,
fit.py:96-131,423-520; see ``diagnostics``). Other reference options raise ``ValueError`` naming
the option.
"""

from __future__ import annotations

import math
from collections.abc import Collection
from dataclasses import dataclass

import numpy as np
import torch

from rtgs_b200 import _native
from rtgs_b200.core.gaussians2d import Gaussians2D
from rtgs_b200.core.metrics import masked_psnr, psnr
from rtgs_b200.image2gs.diagnostics import DiagnosticFit, NativeFitDiagnostic, NativeFitDiagnosticCallback  # noqa: F401
from rtgs_b200.image2gs.engine import FitEngine, acquire_engine, pack_mask_bits, psnr_values, release_engine

_MIN_DIAG = 0.3
_CURRENT_APPEARANCE = "weight_color_9p"
_CANDIDATE_APPEARANCE = "unit_weight_bounded_8p"
_APPEARANCE_PARAMETERIZATIONS = {_CURRENT_APPEARANCE, _CANDIDATE_APPEARANCE}


@dataclass
class FitConfig:
    """Hyperparameters for per-image 2D gaussian fitting (fit.py:31-93, same fields/defaults)."""

    n_gaussians: int = 640
    max_gaussians: int | None = 5_000
    iterations: int = 300
    backend: str = "native"
    adaptive_density: bool = True
    growth_waves: int = 5
    relocate_fraction: float = 0.0
    structsplat_renderer: str = "auto"
    native_renderer: str = "torch"
    batch_views: bool = False
    lr: float = 1e-2
    grad_init_mix: float = 0.7
    init_strategy: str = "gradient"
    structure_sampling: str = "wse"
    row_chunk: int = 64
    log_every: int = 50
    convergence_patience: int = 0
    convergence_tol: float = 0.05
    convergence_check_every: int = 25
    appearance_parameterization: str = _CURRENT_APPEARANCE
    freeze_geometry: bool = False
    pool: bool = False
    pool_capacity: int | None = None
    pool_triage_every: int = 50
    pool_prune_count: int = 32
    pool_spawn_count: int = 32
    pool_min_live: int = 1
    mask_coverage_weight: float = 0.0


class NonFiniteRawParameterError(ValueError):
    """Non-finite native raw parameter (fit.py:134-141)."""

    def __init__(self, parameter_name: str, row_indices: list[int], raw_tensor: torch.Tensor):
        self.parameter_name = parameter_name
        self.row_indices = tuple(row_indices)
        self.raw_tensor = raw_tensor.detach().clone()
        super().__init__(f"non-finite raw rows in {parameter_name}: {row_indices}")


def _softplus_inv(x: torch.Tensor) -> torch.Tensor:
    return x + torch.log(-torch.expm1(-x))


def _gradient_magnitude(image: torch.Tensor) -> torch.Tensor:
    """(H, W) central-difference gradient magnitude of the channel mean (fit.py:148-155)."""
    gray = image.mean(dim=-1)
    gx = torch.zeros_like(gray)
    gy = torch.zeros_like(gray)
    gx[:, 1:-1] = (gray[:, 2:] - gray[:, :-2]) * 0.5
    gy[1:-1, :] = (gray[2:, :] - gray[:-2, :]) * 0.5
    return torch.sqrt(gx**2 + gy**2)


def init_gaussians_2d(
    image: torch.Tensor,
    n: int,
    grad_mix: float = 0.7,
    generator: torch.Generator | None = None,
) -> Gaussians2D:
    """Gradient-magnitude + uniform placement, colours sampled from the image (fit.py:158-187)."""
    h, w = image.shape[:2]
    device = image.device
    grad = _gradient_magnitude(image).reshape(-1)
    uniform = torch.ones_like(grad) / grad.numel()
    prob = grad_mix * grad / grad.sum().clamp_min(1e-8) + (1 - grad_mix) * uniform
    idx = torch.multinomial(prob, n, replacement=True, generator=generator)
    yy = (idx // w).float() + 0.5
    xx = (idx % w).float() + 0.5
    xy = torch.stack([xx, yy], dim=-1)
    xy = xy + (torch.rand(n, 2, generator=generator, device=device) - 0.5)
    xy[:, 0] = xy[:, 0].clamp(0.0, w - 1e-3)
    xy[:, 1] = xy[:, 1].clamp(0.0, h - 1e-3)
    scale0 = max((h * w / n) ** 0.5 * 0.6, _MIN_DIAG + 0.1)
    chol = torch.zeros(n, 3, device=device, dtype=image.dtype)
    chol[:, 0] = scale0
    chol[:, 2] = scale0
    color = image.reshape(-1, 3)[idx].clone()
    weight = torch.full((n,), 0.5, device=device, dtype=image.dtype)
    return Gaussians2D(xy=xy, chol=chol, color=color, weight=weight)


def raw_from_gaussians(xy, chol, color, weight, height: int, width: int,
                       appearance: str = _CURRENT_APPEARANCE) -> dict[str, torch.Tensor]:
    """Raw parameters from constrained ones (fit.py:375-387); works on (..., k) tensors. The
    unit-weight appearance replaces color_raw and weight_raw by
    amplitude_raw = logit(sigmoid(weight_raw) * sigmoid(color_raw))."""
    wh = xy.new_tensor([width, height])
    color_raw = torch.logit(color.clamp(1e-3, 1 - 1e-3))
    weight_raw = torch.logit(weight.clamp(1e-3, 1 - 1e-3))
    raw = {
        "xy_raw": torch.logit((xy / wh).clamp(1e-4, 1 - 1e-4)),
        "diag_raw": _softplus_inv(chol[..., [0, 2]] - _MIN_DIAG),
        "off_raw": chol[..., 1].clone(),
    }
    if appearance == _CANDIDATE_APPEARANCE:
        raw["amplitude_raw"] = torch.logit(torch.sigmoid(weight_raw)[..., None] * torch.sigmoid(color_raw))
    else:
        raw.update(color_raw=color_raw, weight_raw=weight_raw)
    return raw


def _validate_raw_parameters(raw_parameters: dict[str, torch.Tensor]) -> None:
    # One host synchronisation for all fields; the failing rows are gathered only on error.
    finite = {name: torch.isfinite(value) for name, value in raw_parameters.items()}
    if not finite or all(torch.stack([f.all() for f in finite.values()]).tolist()):
        return
    for name, value in raw_parameters.items():
        if bool(finite[name].all()):
            continue
        rows = torch.nonzero(~finite[name].reshape(value.shape[0], -1).all(dim=1)).flatten().tolist()
        raise NonFiniteRawParameterError(name, rows, value)


def _check_initial_shapes(g0: Gaussians2D) -> None:
    """The host-side part of the initialiser checks (fit.py:634-653): shapes and dtypes. The
    reference checks each field's shape, dtype and finiteness in turn, so with a malformed field
    the earlier fields' finiteness decides which error comes first: that case takes the
    field-by-field path."""
    expected = {"xy": (g0.n, 2), "chol": (g0.n, 3), "color": (g0.n, 3), "weight": (g0.n,)}
    for name, shape in expected.items():
        value = getattr(g0, name)
        if not isinstance(value, torch.Tensor) or tuple(value.shape) != shape or not value.is_floating_point():
            for earlier, eshape in expected.items():
                evalue = getattr(g0, earlier)
                if not isinstance(evalue, torch.Tensor) or tuple(evalue.shape) != eshape:
                    actual = None if not isinstance(evalue, torch.Tensor) else tuple(evalue.shape)
                    raise ValueError(f"initial Gaussians2D {earlier} shape must be {eshape}, got {actual}")
                if not evalue.is_floating_point():
                    raise ValueError(f"initial Gaussians2D {earlier} must be floating point")
                finite = torch.isfinite(evalue).reshape(g0.n, -1).all(dim=1)
                if not bool(finite.all()):
                    rows = torch.nonzero(~finite).flatten().tolist()
                    raise ValueError(f"non-finite initial rows in {earlier}: {rows}")


def _validate_initial_gaussians(g0: Gaussians2D, height: int, width: int) -> None:
    """Reject malformed initialiser fields (fit.py:634-676).

    Shapes and dtypes are checked on the host; the value checks run on the device and are read
    back with one synchronisation, and only a failing check gathers its rows, in the reference's
    order of checks (finiteness per field, bounds, Cholesky diagonal, colour / weight range).
    """
    _check_initial_shapes(g0)
    expected = {"xy": (g0.n, 2), "chol": (g0.n, 3), "color": (g0.n, 3), "weight": (g0.n,)}
    finite = {name: torch.isfinite(getattr(g0, name)).reshape(g0.n, -1).all(dim=1) for name in expected}
    inside = (g0.xy[:, 0] >= 0) & (g0.xy[:, 0] < width) & (g0.xy[:, 1] >= 0) & (g0.xy[:, 1] < height)
    diag_ok = (g0.chol[:, 0] > _MIN_DIAG) & (g0.chol[:, 2] > _MIN_DIAG)
    unit = {name: ((getattr(g0, name) >= 0) & (getattr(g0, name) <= 1)).reshape(g0.n, -1).all(dim=1)
            for name in ("color", "weight")}
    checks = [*finite.values(), inside, diag_ok, *unit.values()]
    if all(torch.stack([c.all() for c in checks]).tolist()):
        return
    for name in expected:
        if not bool(finite[name].all()):
            rows = torch.nonzero(~finite[name]).flatten().tolist()
            raise ValueError(f"non-finite initial rows in {name}: {rows}")
    if not bool(inside.all()):
        rows = torch.nonzero(~inside).flatten().tolist()
        raise ValueError(f"initial Gaussians2D xy rows outside image bounds: {rows}")
    if not bool(diag_ok.all()):
        rows = torch.nonzero(~diag_ok).flatten().tolist()
        raise ValueError(f"initial Gaussians2D Cholesky diagonal must exceed {_MIN_DIAG}: rows {rows}")
    for name, ok in unit.items():
        if not bool(ok.all()):
            rows = torch.nonzero(~ok).flatten().tolist()
            raise ValueError(f"initial Gaussians2D {name} rows outside [0,1]: {rows}")


def _validate_fit_controls(config: FitConfig, diagnostic_callback=None, diagnostic_steps: Collection[int] = ()) -> None:
    """Reference validation (fit.py:575-622) plus the options this package does not implement."""
    if config.appearance_parameterization not in _APPEARANCE_PARAMETERIZATIONS:
        choices = ", ".join(sorted(_APPEARANCE_PARAMETERIZATIONS))
        raise ValueError(f"appearance_parameterization must be one of: {choices}")
    if config.native_renderer not in ("torch", "cuda", "auto"):
        raise ValueError("native_renderer must be 'torch', 'cuda', or 'auto'")
    if config.init_strategy not in ("gradient", "structure_tensor"):
        raise ValueError("init_strategy must be 'gradient' or 'structure_tensor'")
    if config.structure_sampling not in ("wse", "density"):
        raise ValueError("structure_sampling must be 'wse' or 'density'")
    if config.init_strategy != "structure_tensor" and config.structure_sampling != "wse":
        raise ValueError("structure_sampling='density' requires init_strategy='structure_tensor'")
    steps = tuple(diagnostic_steps)  # fit.py:593-599
    if diagnostic_callback is None and steps:
        raise ValueError("diagnostic_steps require diagnostic_callback")
    if any(isinstance(step, bool) or not isinstance(step, int) for step in steps):
        raise ValueError("diagnostic_steps must contain integers")
    if any(step < 0 or step > config.iterations for step in steps):
        raise ValueError("diagnostic_steps must lie in [0, iterations]")
    if config.mask_coverage_weight < 0.0:
        raise ValueError("mask_coverage_weight must be non-negative")
    if config.backend != "native":
        raise ValueError("fit backend must be 'native' (StructSplat is not part of this package)")
    if config.init_strategy != "gradient":
        raise ValueError("init_strategy='structure_tensor' is not implemented by rtgs_b200")
    if config.pool:  # fit.py:600-616
        if config.appearance_parameterization != _CURRENT_APPEARANCE:
            raise ValueError("pool fitting supports only the default appearance parameterization")
        if config.freeze_geometry:
            raise ValueError("pool fitting is incompatible with freeze_geometry")
        if diagnostic_callback is not None or tuple(diagnostic_steps):
            raise ValueError("pool fitting does not support native fit diagnostics")
        if config.pool_capacity is not None and config.pool_capacity < config.n_gaussians:
            raise ValueError("pool_capacity must be at least n_gaussians")
        if config.pool_min_live < 1:
            raise ValueError("pool_min_live must be at least 1")
        for name in ("pool_triage_every", "pool_prune_count", "pool_spawn_count"):
            if getattr(config, name) < 0:
                raise ValueError(f"{name} must be non-negative")
    if config.mask_coverage_weight > 0.0 and (config.batch_views or config.pool):  # fit.py:618-622
        raise ValueError("mask_coverage_weight is not supported with batch_views or the pool")
    if config.iterations < 1:
        raise ValueError("iterations must be >= 1")


def _crop_to_mask(image: torch.Tensor, mask: torch.Tensor, margin_fraction: float = 0.05):
    """Crop a masked fit to the foreground bbox + margin; returns the xy offset (fit.py:792-807)."""
    if mask.shape != image.shape[:2]:
        raise ValueError("mask size does not match image")
    foreground = torch.nonzero(mask > 0.5)
    if foreground.numel() == 0:
        raise ValueError("cannot fit an empty foreground mask")
    height, width = image.shape[:2]
    margin = max(2, round(max(height, width) * margin_fraction))
    y0 = max(0, int(foreground[:, 0].min()) - margin)
    y1 = min(height, int(foreground[:, 0].max()) + 1 + margin)
    x0 = max(0, int(foreground[:, 1].min()) - margin)
    x1 = min(width, int(foreground[:, 1].max()) + 1 + margin)
    return image[y0:y1, x0:x1], mask[y0:y1, x0:x1], image.new_tensor([x0, y0])


def _require_cuda(image: torch.Tensor) -> None:
    if not image.is_cuda:
        raise RuntimeError(
            "the rtgs stage-1 CUDA renderer requires CUDA tensors; move the fit to a CUDA device"
        )


def _history_from_engine(engine: FitEngine, config: FitConfig, counts: np.ndarray) -> list[dict]:
    iters, sums = engine.history()
    out = [{"psnr": [], "stopped_iter": config.iterations - 1} for _ in range(engine.n_views)]
    for r, it in enumerate(iters):
        it = int(it)
        if it % config.log_every == 0 or it == config.iterations - 1:
            vals = psnr_values(sums[r, :, 1], counts)
            for b in range(engine.n_views):
                out[b]["psnr"].append((it, vals[b]))
    return out


def _fit_native_from_initialization(
    image: torch.Tensor,
    target: torch.Tensor,
    g0: Gaussians2D,
    config: FitConfig,
    mask: torch.Tensor | None,
    xy_offset: torch.Tensor,
    diagnostic_callback: NativeFitDiagnosticCallback | None = None,
    diagnostic_steps: Collection[int] = (),
    initializer_rng_state_before: torch.Tensor | None = None,
    initializer_rng_state_after: torch.Tensor | None = None,
) -> tuple[Gaussians2D, dict]:
    """Device fit loop for one image (fit.py:355-554).

    The initialiser's value checks and raw transform run in one engine call
    (``FitEngine.set_initial``); only when a check fails are the torch checks run, to report the
    failing rows with the reference's messages. With a ``diagnostic_callback`` the loop runs one
    iteration at a time and emits the reference's snapshots (``diagnostics.DiagnosticFit``).
    """
    _require_cuda(image)
    h, w = image.shape[:2]
    _check_initial_shapes(g0)
    if config.mask_coverage_weight > 0.0 and mask is None:  # fit.py:371-372
        raise ValueError("mask_coverage_weight requires a mask")
    loss_mode = _native.LOSS_MSE if mask is None else _native.LOSS_MASK_WEIGHTED
    patience = int(config.convergence_patience)
    check_every = int(config.convergence_check_every) if patience else 0
    engine = acquire_engine(
        1, g0.n, h, w, lr=config.lr, iterations=config.iterations, log_every=config.log_every,
        check_every=check_every, freeze_geometry=config.freeze_geometry, loss_mode=loss_mode,
        device=image.device, mask_coverage_weight=config.mask_coverage_weight if mask is not None else 0.0,
        appearance=config.appearance_parameterization,
    )
    ok = False
    try:
        status = engine.set_initial(g0.xy, g0.chol, g0.color, g0.weight)
        if status:
            ok = True  # the engine itself is fine: keep it pooled
            _raise_initial_errors(g0, h, w, config.appearance_parameterization)
        ok = False
        mask_bits = None if mask is None else pack_mask_bits(mask[None])
        engine.set_targets(target[None], mask_bits)
        counts = np.array([3.0 * h * w])
        stopped = config.iterations - 1
        if diagnostic_callback is not None:
            coverage_fn = None
            if config.mask_coverage_weight > 0.0 and mask is not None:
                from rtgs_b200.image2gs.renderer2d import render_gaussian_coverage_2d

                outside = 1.0 - mask.to(target).clamp(0, 1)

                def coverage_fn(g: Gaussians2D) -> torch.Tensor:  # fit.py:566-572
                    return config.mask_coverage_weight * (render_gaussian_coverage_2d(g, h, w) * outside).mean()

            stopped = DiagnosticFit(
                engine, config=config, g0=g0, target=target, mask=mask, callback=diagnostic_callback,
                steps=diagnostic_steps, rng_state_before=initializer_rng_state_before,
                rng_state_after=initializer_rng_state_after, coverage_fn=coverage_fn,
            ).run(counts, patience, check_every, config.convergence_tol)
        elif patience:
            best, stale = -float("inf"), 0
            done = 0
            while done < config.iterations:
                chunk = min(check_every - (done % check_every), config.iterations - done)
                engine.run(chunk)
                done += chunk
                if done % check_every == 0:
                    iters, sums = engine.history()
                    cur = psnr_values(sums[-1, :, 1], counts)[0]
                    if cur > best + config.convergence_tol:
                        best, stale = cur, 0
                    else:
                        stale += 1
                        if stale >= patience:
                            stopped = done - 1
                            break
        else:
            engine.run(config.iterations)
        history = _history_from_engine(engine, config, counts)[0]
        if stopped != config.iterations - 1:
            # The reference logs the stopping iteration only if it is a log step.
            history["psnr"] = [(i, v) for i, v in history["psnr"] if i <= stopped]
            history["stopped_iter"] = stopped
        xy, chol, color, weight = (t[0] for t in engine.params())
        # Unmasked: the final PSNR from the evaluation's clamped squared-error sum (no render is
        # materialised); masked: masked_psnr of the render against the uncropped-mask image.
        final, sums = engine.evaluate(want_render=mask is not None)
        ok = True
    finally:
        release_engine(engine, reusable=ok)
    result = Gaussians2D(xy=xy, chol=chol, color=color, weight=weight)
    if mask is None:
        history["final_psnr_full"] = psnr_values(sums[:, 1], counts)[0]
        history["final_psnr"] = history["final_psnr_full"]
    else:
        pred = final[0].clamp(0, 1)
        history["final_psnr_full"] = psnr(pred, target)
        history["final_psnr"] = masked_psnr(pred, image, mask)
    result.xy += xy_offset
    return result, history


def _raise_initial_errors(g0: Gaussians2D, height: int, width: int,
                          appearance: str = _CURRENT_APPEARANCE) -> None:
    """An initialisation the engine rejected: raise the reference's error for it (fit.py:634-676,
    then fit.py:134-141 for non-finite raw parameters)."""
    _validate_initial_gaussians(g0, height, width)
    _validate_raw_parameters(raw_from_gaussians(g0.xy, g0.chol, g0.color, g0.weight, height, width, appearance))
    raise RuntimeError("the engine rejected the initial gaussians but no check fails on the host")


def fit_image(
    image: torch.Tensor,
    config: FitConfig | None = None,
    seed: int | None = None,
    mask: torch.Tensor | None = None,
    *,
    diagnostic_callback=None,
    diagnostic_steps: Collection[int] = (),
    observation_callback=None,
    observation_view_id: str | None = None,
) -> tuple[Gaussians2D, dict]:
    """Fit 2D gaussians to an (H, W, 3) CUDA image in [0,1] (fit.py:222-306)."""
    config = config or FitConfig()
    _validate_fit_controls(config, diagnostic_callback, diagnostic_steps)
    if observation_callback is not None or observation_view_id is not None:
        raise ValueError("lossless observation export currently requires the StructSplat backend")
    _require_cuda(image)
    xy_offset = image.new_zeros(2)
    if mask is not None:
        image, mask, xy_offset = _crop_to_mask(image, mask)
    target = image
    if mask is not None:
        target = image * mask.to(image).clamp(0, 1)[..., None]
    gen = None
    rng_state_before = rng_state_after = None
    if seed is not None:
        gen = torch.Generator(device=image.device).manual_seed(seed)
        if diagnostic_callback is not None:
            rng_state_before = gen.get_state().clone()
    g0 = init_gaussians_2d(target, config.n_gaussians, config.grad_init_mix, gen)
    if diagnostic_callback is not None and gen is not None:
        rng_state_after = gen.get_state().clone()
    if config.pool:
        from rtgs_b200.image2gs.pool import fit_pooled_from_initialization

        return fit_pooled_from_initialization(image, target, g0, config, mask, xy_offset)
    return _fit_native_from_initialization(
        image, target, g0, config, mask, xy_offset, diagnostic_callback=diagnostic_callback,
        diagnostic_steps=diagnostic_steps, initializer_rng_state_before=rng_state_before,
        initializer_rng_state_after=rng_state_after,
    )


def fit_image_from_initialization(
    image: torch.Tensor,
    initial_gaussians: Gaussians2D,
    config: FitConfig | None = None,
    mask: torch.Tensor | None = None,
    *,
    diagnostic_callback=None,
    diagnostic_steps: Collection[int] = (),
) -> tuple[Gaussians2D, dict]:
    """Fit from a supplied initialisation (fit.py:309-352)."""
    config = config or FitConfig()
    _validate_fit_controls(config, diagnostic_callback, diagnostic_steps)
    _require_cuda(image)
    xy_offset = image.new_zeros(2)
    if mask is not None:
        image, mask, xy_offset = _crop_to_mask(image, mask)
    target = image
    if mask is not None:
        target = image * mask.to(image).clamp(0, 1)[..., None]
    g0 = initial_gaussians.to(image.device)
    if config.pool:
        from rtgs_b200.image2gs.pool import fit_pooled_from_initialization

        return fit_pooled_from_initialization(image, target, g0, config, mask, xy_offset)
    return _fit_native_from_initialization(image, target, g0, config, mask, xy_offset,
                                           diagnostic_callback=diagnostic_callback,
                                           diagnostic_steps=diagnostic_steps)


def fit_views(
    images: list[torch.Tensor],
    config: FitConfig | None = None,
    seed: int = 0,
    masks: list[torch.Tensor] | None = None,
) -> tuple[list[Gaussians2D], list[dict]]:
    """Fit every view independently, or jointly with ``config.batch_views`` (fit.py:768-789)."""
    if config is not None and config.batch_views:
        from rtgs_b200.image2gs.batched import fit_views_batched

        return fit_views_batched(images, config, seed=seed, masks=masks)
    results, histories = [], []
    for i, image in enumerate(images):
        mask = None if masks is None else masks[i]
        g, hist = fit_image(image, config, seed=seed + i, mask=mask)
        results.append(g)
        histories.append(hist)
    return results, histories


def psnr_from_sums(sse: float, count: float) -> float:
    mse = max(sse / count, 1e-12)
    return -10.0 * math.log10(mse)
