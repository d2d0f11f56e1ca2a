"""Differentiable accumulated 2D gaussian splatting (reference: src/rtgs/image2gs/renderer2d.py).

Pixel colour is ``sum_i weight_i * color_i * exp(-0.5 d^T Sigma_i^-1 d)`` over the gaussians whose
support rectangle (Mahalanobis cutoff 12, renderer2d.py:156-181) contains the pixel and whose
q = d^T Sigma^-1 d is below 12; pixel centres are at (x + 0.5, y + 0.5).

Same entry points and argument validation as the reference. This package has exactly one
implementation, the sm_100a kernels of librtgs2d: ``renderer`` is accepted for compatibility and
validated like the reference (``ValueError`` for unknown names), and every accepted value runs
the CUDA kernels. CPU tensors raise ``RuntimeError`` (there is no CPU fallback); ``row_chunk``
only bounded the reference's CPU memory and is accepted and ignored.
"""

from __future__ import annotations

import torch

from rtgs_b200.core.gaussians2d import Gaussians2D

_CUTOFF = 12.0
_RENDERERS = ("torch", "cuda", "auto")


def _resolve_renderer(renderer: str, device: torch.device) -> str:
    if renderer not in _RENDERERS:
        raise ValueError(f"renderer must be one of {_RENDERERS}, got {renderer!r}")
    return "cuda"


def render_gaussians_2d(
    g: Gaussians2D,
    height: int,
    width: int,
    background: torch.Tensor | None = None,
    row_chunk: int = 64,
    renderer: str = "torch",
) -> torch.Tensor:
    """Render 2D gaussians to an (H, W, 3) image, differentiably (renderer2d.py:37-69)."""
    _resolve_renderer(renderer, g.xy.device)
    return render_gaussians_2d_batched(
        g.xy[None], g.chol[None], g.color[None], g.weight[None], height, width,
        background=background, row_chunk=row_chunk, renderer=renderer,
    )[0]


def render_gaussians_2d_batched(
    xy: torch.Tensor,
    chol: torch.Tensor,
    color: torch.Tensor,
    weight: torch.Tensor,
    height: int,
    width: int,
    background: torch.Tensor | None = None,
    row_chunk: int = 64,
    renderer: str = "torch",
) -> torch.Tensor:
    """Render B stacked same-sized views to (B, H, W, 3) in one pass (renderer2d.py:72-125)."""
    if xy.dim() != 3 or xy.shape[-1] != 2:
        raise ValueError("batched xy must be (B, N, 2)")
    n_views, n = xy.shape[:2]
    if chol.shape != (n_views, n, 3) or color.shape != (n_views, n, 3):
        raise ValueError("batched chol/color must be (B, N, 3)")
    if weight.shape != (n_views, n):
        raise ValueError("batched weight must be (B, N)")
    _resolve_renderer(renderer, xy.device)
    from rtgs_b200.image2gs.cuda_backend import render_batched_cuda

    img = render_batched_cuda(xy, chol, color, weight, height, width)
    if background is not None:
        img = img + background.to(img)[None, None, None, :]
    return img


def render_gaussian_coverage_2d(
    g: Gaussians2D,
    height: int,
    width: int,
    row_chunk: int = 64,
) -> torch.Tensor:
    """Colour-independent soft coverage ``1 - exp(-sum_i weight_i G_i)`` (renderer2d.py:128-140)."""
    from rtgs_b200.image2gs.cuda_backend import render_batched_cuda_with_density

    _, density = render_batched_cuda_with_density(
        g.xy[None], g.chol[None], g.color[None], g.weight[None], height, width
    )
    return 1.0 - torch.exp(-density[0])
