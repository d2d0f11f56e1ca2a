"""Image metrics on (H, W, 3) float tensors in [0, 1] (reference: src/rtgs/core/metrics.py:12-29)."""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def psnr(pred: torch.Tensor, target: torch.Tensor) -> float:
    """Peak signal-to-noise ratio in dB (max value 1.0)."""
    mse = F.mse_loss(pred, target).clamp_min(1e-12)
    return float(-10.0 * torch.log10(mse))


def masked_psnr(pred: torch.Tensor, target: torch.Tensor, mask: torch.Tensor) -> float:
    """Foreground-weighted PSNR (mean over mask pixels x 3 channels)."""
    if pred.shape != target.shape or pred.ndim != 3 or pred.shape[-1] != 3:
        raise ValueError("pred and target must have matching (H, W, 3) shapes")
    if mask.shape != pred.shape[:2]:
        raise ValueError("mask must match the image height and width")
    weights = mask.to(device=pred.device, dtype=pred.dtype).clamp(0, 1)
    if not bool(weights.sum() > 0):
        raise ValueError("mask has no foreground pixels")
    denominator = weights.sum() * pred.shape[-1]
    mse = (((pred - target) ** 2) * weights[..., None]).sum() / denominator
    return float(-10.0 * torch.log10(mse.clamp_min(1e-12)))


def psnr_from_sse(sse: float, count: float) -> float:
    """PSNR from a sum of squared errors over `count` values (same clamp as ``psnr``)."""
    mse = max(sse / count, 1e-12) if count > 0 else 1e-12
    return -10.0 * math.log10(mse)
