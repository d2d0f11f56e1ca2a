"""Helpers shared by the GPU parity tests (device inputs, C-ABI calls, oracle references)."""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from oracle import render2d as orender
from rtgs_b200 import _native

DEV = torch.device("cuda", 0)


def stacked(seed: int, n_views: int, n: int, height: int, width: int, margin: float = 4.0,
            lo: float = 0.5, hi: float = 3.5, off: float = 0.5):
    """Random stacked gaussians incl. off-image and edge-straddling centres (CPU tensors)."""
    gen = torch.Generator().manual_seed(seed)
    span = torch.tensor([width + 2 * margin, height + 2 * margin])
    xy = torch.rand(n_views, n, 2, generator=gen) * span - margin
    chol = torch.zeros(n_views, n, 3)
    chol[..., 0] = lo + (hi - lo) * torch.rand(n_views, n, generator=gen)
    chol[..., 2] = lo + (hi - lo) * torch.rand(n_views, n, generator=gen)
    chol[..., 1] = off * torch.randn(n_views, n, generator=gen)
    color = torch.rand(n_views, n, 3, generator=gen)
    weight = torch.rand(n_views, n, generator=gen)
    return xy, chol, color, weight


def cuda(*ts):
    return tuple(x.to(DEV).contiguous() for x in ts)


def support_rects(xy: torch.Tensor, chol: torch.Tensor, height: int, width: int):
    """Device rectangles + pixel counts through the C ABI (rtgs2d_support_rects)."""
    m = xy.shape[0]
    rects = torch.empty(m, 4, dtype=torch.int32, device=DEV)
    counts = torch.empty(m, dtype=torch.int64, device=DEV)
    xy, chol = cuda(xy.reshape(-1, 2), chol.reshape(-1, 3))
    _native.check(_native.lib().rtgs2d_support_rects(xy.data_ptr(), chol.data_ptr(), m, height, width,
                                                     rects.data_ptr(), counts.data_ptr(),
                                                     _native.stream_ptr(DEV)))
    torch.cuda.synchronize()
    return rects.cpu(), counts.cpu()


def last_binning():
    """(gids, ranges) of the last render on device 0's arena, copied through the C ABI."""
    lib = _native.lib()
    n_e, n_t = ctypes.c_int64(), ctypes.c_int64()
    a = _native.arena(DEV)
    _native.check(lib.rtgs2d_arena_copy_binning(a, 0, None, 0, None, ctypes.byref(n_e), ctypes.byref(n_t), None))
    gids = np.zeros(max(n_e.value, 1), dtype=np.uint32)
    ranges = np.zeros((max(n_t.value, 1), 2), dtype=np.int32)
    _native.check(lib.rtgs2d_arena_copy_binning(a, n_e.value, gids.ctypes.data, n_t.value, ranges.ctypes.data,
                                                ctypes.byref(n_e), ctypes.byref(n_t), None))
    return gids[: n_e.value], ranges[: n_t.value]


def oracle_render(xy, chol, color, weight, height, width, with_density=False):
    return orender.render_batched(xy.cpu(), chol.cpu(), color.cpu(), weight.cpu(), height, width,
                                  with_density=with_density)


def oracle_grads(xy, chol, color, weight, height, width, up, up_den=None, accumulate_dtype=None):
    """Oracle gradients of sum(render * up) (+ sum(density * up_den)); with
    ``accumulate_dtype=torch.float64`` the reference's float32 support set with float64 sums."""
    leaves = [x.detach().cpu().clone().requires_grad_(True) for x in (xy, chol, color, weight)]
    img, den = orender.render_batched(*leaves, height, width, with_density=True, accumulate_dtype=accumulate_dtype)
    if accumulate_dtype is not None:
        up = up.to(accumulate_dtype)
        up_den = None if up_den is None else up_den.to(accumulate_dtype)
    loss = (img * up.cpu()).sum()
    if up_den is not None:
        loss = loss + (den * up_den.cpu()).sum()
    loss.backward()
    return [leaf.grad if leaf.grad is not None else torch.zeros_like(leaf) for leaf in leaves]
