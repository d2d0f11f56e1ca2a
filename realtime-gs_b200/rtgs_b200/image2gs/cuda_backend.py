"""sm_100a backend of the batched Stage-1 renderer (reference: src/rtgs/image2gs/cuda_backend.py).

``render_batched_cuda(xy, chol, color, weight, H, W)`` keeps the reference signature and error
messages (cuda_backend.py:127-170). Unlike the reference, conics, support rectangles and tile
binning are computed on the device by librtgs2d, gradients flow to ``chol`` through a fused
conic -> Cholesky chain rule instead of torch ops, and results are deterministic (tile lists in
gaussian order, fixed-order gradient reduction; the reference accumulated with atomics).

Nothing here touches CUDA at import time (reference rule, cuda_backend.py:9-10).
"""

from __future__ import annotations

import torch
from torch.autograd import Function
from torch.autograd.function import once_differentiable

from rtgs_b200 import _native

_CUTOFF = 12.0


def _check_inputs(xy: torch.Tensor, chol: torch.Tensor, color: torch.Tensor, weight: torch.Tensor) -> None:
    if not xy.is_cuda or not chol.is_cuda or not color.is_cuda or not weight.is_cuda:
        raise RuntimeError(
            "the rtgs stage-1 CUDA renderer requires CUDA tensors; "
            "move the fit to a CUDA device"
        )
    if any(t.dtype != torch.float32 for t in (xy, chol, color, weight)):
        raise RuntimeError("the rtgs stage-1 CUDA renderer supports float32 tensors only")
    devices = {t.device for t in (xy, chol, color, weight)}
    if len(devices) != 1:
        raise RuntimeError("the rtgs stage-1 CUDA renderer needs all tensors on one device")


def _forward(xy, chol, color, weight, height: int, width: int, want_den: bool):
    n_views, n = xy.shape[:2]
    device = xy.device
    out = torch.empty((n_views, height, width, 3), device=device, dtype=torch.float32)
    den = torch.empty((n_views, height, width), device=device, dtype=torch.float32) if want_den else None
    L = _native.lib()
    with torch.cuda.device(device):
        _native.check(
            L.rtgs2d_render_forward(
                _native.arena(device), xy.data_ptr(), chol.data_ptr(), color.data_ptr(),
                weight.data_ptr(), n_views, n, height, width, out.data_ptr(), _native.ptr(den),
                _native.stream_ptr(device),
            )
        )
    return out, den


def _backward(ctx, grad_out, grad_den):
    xy, chol, color, weight = ctx.saved_tensors
    height, width = ctx.dims
    need = ctx.needs_input_grad[:4]
    if not any(need):
        return None, None, None, None
    n_views, n = xy.shape[:2]
    grads = [torch.empty_like(t) if want else None for t, want in zip((xy, chol, color, weight), need)]
    device = xy.device
    go = grad_out.contiguous() if grad_out is not None else None
    gd = grad_den.contiguous() if grad_den is not None else None
    L = _native.lib()
    with torch.cuda.device(device):
        # Saved tensors are alive and unmodified (autograd enforces it), so the forward's
        # binning is reused when nothing else has binned on the arena since.
        _native.check(
            L.rtgs2d_render_backward_after_forward(
                _native.arena(device), _native.ptr(go), _native.ptr(gd), xy.data_ptr(),
                chol.data_ptr(), color.data_ptr(), weight.data_ptr(), n_views, n, height, width,
                *(_native.ptr(g) for g in grads), _native.stream_ptr(device),
            )
        )
    return tuple(grads)


class _Render2DBatched(Function):
    @staticmethod
    def forward(ctx, xy, chol, color, weight, height, width):
        out, _ = _forward(xy, chol, color, weight, height, width, False)
        ctx.save_for_backward(xy, chol, color, weight)
        ctx.dims = (int(height), int(width))
        return out

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_out):
        return (*_backward(ctx, grad_out, None), None, None)


class _Render2DBatchedDensity(Function):
    @staticmethod
    def forward(ctx, xy, chol, color, weight, height, width):
        out, den = _forward(xy, chol, color, weight, height, width, True)
        ctx.save_for_backward(xy, chol, color, weight)
        ctx.dims = (int(height), int(width))
        return out, den

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_out, grad_den):
        return (*_backward(ctx, grad_out, grad_den), None, None)


def _prepare(xy, chol, color, weight):
    _check_inputs(xy, chol, color, weight)
    return xy.contiguous(), chol.contiguous(), color.contiguous(), weight.contiguous()


def render_batched_cuda(
    xy: torch.Tensor,
    chol: torch.Tensor,
    color: torch.Tensor,
    weight: torch.Tensor,
    height: int,
    width: int,
) -> torch.Tensor:
    """Render (B, N) stacked gaussians to (B, H, W, 3) (cuda_backend.py:127-170).

    Shapes are validated by the ``renderer2d`` caller; this checks device and dtype only.
    Differentiable with respect to all four inputs.
    """
    xy, chol, color, weight = _prepare(xy, chol, color, weight)
    return _Render2DBatched.apply(xy, chol, color, weight, int(height), int(width))


def render_batched_cuda_with_density(
    xy: torch.Tensor,
    chol: torch.Tensor,
    color: torch.Tensor,
    weight: torch.Tensor,
    height: int,
    width: int,
) -> tuple[torch.Tensor, torch.Tensor]:
    """(B, H, W, 3) image and (B, H, W) density sum_i weight_i G_i, both differentiable."""
    xy, chol, color, weight = _prepare(xy, chol, color, weight)
    return _Render2DBatchedDensity.apply(xy, chol, color, weight, int(height), int(width))


def last_render_stats(device: torch.device | None = None) -> tuple[int, int]:
    """(tile entries, pixel pairs) of the last render/backward on `device`'s arena."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    return _native.arena_last_stats(device)
