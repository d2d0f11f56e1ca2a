"""CPU oracle: accumulated (additive) 2D gaussian splatting, restated from the reference.

TEST INFRASTRUCTURE ONLY -- imported by tests/, __graft_entry__.smoke() and bench.py's CPU
baseline leg; never by the product package.

Restated reference behaviour (paths relative to the reference project):
  - covariance Sigma = L L^T            src/rtgs/core/gaussians2d.py:21-31
  - analytic inverse covariance         src/rtgs/core/gaussians2d.py:34-44
  - support rectangles                  src/rtgs/image2gs/renderer2d.py:156-181
  - flat scatter accumulation           src/rtgs/image2gs/renderer2d.py:205-254
  - batched entry + view offsets        src/rtgs/image2gs/renderer2d.py:72-125
  - CUDA-path input conventions         src/rtgs/image2gs/cuda_backend.py:151-158 (rects with
                                        x1 = x0 - 1 when empty) and
                                        src/rtgs/image2gs/cuda/renderer2d_ext.cu:54-58,75-77
                                        (non-finite means and non-finite q contribute nothing)

The arithmetic keeps the reference's float32 operation order: every product and sum is a separate
torch op, so each intermediate is rounded exactly as in the reference. Two deliberate choices
follow the reference's CUDA path rather than its torch path, because that is the contract the
drop-in replaces: a gaussian with a non-finite mean is dropped, and a pair whose q is not finite
contributes zero (the torch path would spread NaN through ``exp(nan) * 0``).
"""

from __future__ import annotations

import numpy as np
import torch

CUTOFF = 12.0
TILE = 16
DEFAULT_BUDGET = 1 << 20  # pairs per index_add chunk in tests (large chunks run fastest here)


def reference_budget(width: int, row_chunk: int = 64) -> int:
    """Pairs per index_add chunk in the reference's torch renderer: max(row_chunk * width, 65536)
    (renderer2d.py:227) with FitConfig.row_chunk = 64 (fit.py:65). Every chunk adds into a new copy
    of the whole frame, so the chunk size sets much of the reference's CPU time: the CPU baselines
    time the oracle with this budget. Renders do not depend on it; gradients only to float32
    rounding (the order of autograd's scatter-add over a gaussian's pairs)."""
    return max(int(row_chunk) * int(width), 65_536)


def chol_covariance(chol: torch.Tensor) -> torch.Tensor:
    """(..., 2, 2) Sigma = L L^T with the reference's rounding (no fused multiply-add)."""
    l11, l21, l22 = chol[..., 0], chol[..., 1], chol[..., 2]
    s00 = l11 * l11
    s01 = l11 * l21
    s11 = (l21 * l21) + (l22 * l22)
    return torch.stack([torch.stack([s00, s01], -1), torch.stack([s01, s11], -1)], dim=-2)


def chol_conics(chol: torch.Tensor) -> torch.Tensor:
    """(..., 3) inverse-covariance entries (i00, i01, i11) from packed (l11, l21, l22)."""
    l11, l21, l22 = chol[..., 0], chol[..., 1], chol[..., 2]
    a = torch.reciprocal(l11)
    b = -l21 / (l11 * l22)
    c = torch.reciprocal(l22)
    return torch.stack([a * a + b * b, b * c, c * c], dim=-1)


def _to_index(v: torch.Tensor) -> torch.Tensor:
    """float -> int64 like the reference's ``.long()`` on x86: NaN/inf/out-of-range -> INT64_MIN."""
    ok = torch.isfinite(v) & (v.abs() < 2.0**63)
    return torch.where(ok, v, torch.zeros_like(v)).long().masked_fill(~ok, -(2**63))


def support_rects(xy: torch.Tensor, cov: torch.Tensor, height: int, width: int):
    """(x0, x1, y0, y1, counts) int64, like renderer2d.py:156-181 (inputs detached)."""
    rx = (CUTOFF * cov[:, 0, 0].clamp_min(0)).sqrt()
    ry = (CUTOFF * cov[:, 1, 1].clamp_min(0)).sqrt()
    x, y = xy[:, 0], xy[:, 1]
    x0 = _to_index(torch.ceil(x - rx - 0.5)).clamp(0, width - 1)
    x1 = _to_index(torch.floor(x + rx - 0.5)).clamp(0, width - 1)
    y0 = _to_index(torch.ceil(y - ry - 0.5)).clamp(0, height - 1)
    y1 = _to_index(torch.floor(y + ry - 0.5)).clamp(0, height - 1)
    outside = (x + rx < 0.5) | (x - rx > width - 0.5) | (y + ry < 0.5) | (y - ry > height - 0.5)
    nx = (x1 - x0 + 1).clamp_min(0)
    ny = (y1 - y0 + 1).clamp_min(0)
    counts = torch.where(outside, torch.zeros_like(nx), nx * ny)
    return x0, x1, y0, y1, counts


def cuda_rects(xy: torch.Tensor, chol: torch.Tensor, height: int, width: int) -> torch.Tensor:
    """(M, 4) int32 (x0, x1, y0, y1) with x1 = x0 - 1 for empty support (cuda_backend.py:153-158)."""
    with torch.no_grad():
        x0, x1, y0, y1, counts = support_rects(xy.detach(), chol_covariance(chol.detach()), height, width)
        x1 = torch.where(counts > 0, x1, x0 - 1)
        return torch.stack([x0, x1, y0, y1], dim=-1).int()


def accumulate(
    xy: torch.Tensor,
    conics: torch.Tensor,
    color: torch.Tensor,
    weight: torch.Tensor,
    rects: torch.Tensor,
    view_index: torch.Tensor,
    n_views: int,
    height: int,
    width: int,
    budget: int = DEFAULT_BUDGET,
    origin: tuple[int, int] = (0, 0),
    support_inputs: tuple[torch.Tensor, torch.Tensor] | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Scatter-add every (gaussian, pixel-in-rect) pair; returns flat color sums and densities.

    Pairs are enumerated gaussian by gaussian in ascending index and, inside a rectangle, row by
    row; ``index_add`` then sums each pixel in that order (renderer2d.py:228-253). Differentiable
    with respect to xy, conics, color and weight through torch autograd, as in the reference.

    ``origin`` = (x, y) renders a window of a larger frame: pixel coordinates (and rectangles)
    stay those of the frame, the outputs hold the ``height`` x ``width`` window starting at the
    origin, and the rectangles must lie inside that window.

    ``support_inputs`` = (xy, conics) computes q from those tensors instead, for the support test
    and the pair's value exp(-q/2), while the gradient follows q of the differentiable inputs:
    with float32 support inputs and float64 differentiable inputs, every pair has the float32
    reference's value and the sums are exact to float64.
    """
    dtype = xy.dtype
    n_pix = n_views * height * width
    color_sum = torch.zeros(n_pix, 3, dtype=dtype)
    density = torch.zeros(n_pix, dtype=dtype)
    with torch.no_grad():
        x0 = rects[:, 0].long()
        y0 = rects[:, 2].long()
        nx = (rects[:, 1].long() - x0 + 1).clamp_min(0)
        ny = (rects[:, 3].long() - y0 + 1).clamp_min(0)
        finite = torch.isfinite(xy.detach()).all(dim=1)
        counts = torch.where(finite, nx * ny, torch.zeros_like(nx))
        csum = counts.cumsum(0)
    m = xy.shape[0]
    start = 0
    while start < m:
        base = int(csum[start - 1]) if start > 0 else 0
        end = int(torch.searchsorted(csum, base + budget, right=True))
        end = max(start + 1, min(end, m))
        local = counts[start:end]
        total = int(local.sum())
        if total:
            with torch.no_grad():
                lid = torch.repeat_interleave(torch.arange(end - start), local)
                gid = lid + start
                first = local.cumsum(0) - local
                off = torch.arange(total) - first[lid]
                px = x0[gid] + off % nx[gid]
                py = y0[gid] + off // nx[gid]
                flat = view_index[gid].long() * (height * width) + (py - origin[1]) * width + (px - origin[0])
            dx = (px.to(dtype) + 0.5) - xy[gid, 0]
            dy = (py.to(dtype) + 0.5) - xy[gid, 1]
            q = ((dx * dx) * conics[gid, 0] + ((2.0 * dx) * dy) * conics[gid, 1]) + (
                dy * dy
            ) * conics[gid, 2]
            if support_inputs is None:
                support = q < CUTOFF
            else:
                with torch.no_grad():
                    s_xy, s_con = support_inputs
                    sdx = (px.to(s_xy.dtype) + 0.5) - s_xy[gid, 0]
                    sdy = (py.to(s_xy.dtype) + 0.5) - s_xy[gid, 1]
                    sq = ((sdx * sdx) * s_con[gid, 0] + ((2.0 * sdx) * sdy) * s_con[gid, 1]) + (
                        sdy * sdy
                    ) * s_con[gid, 2]
                    support = sq < CUTOFF
                # The pair's value is the reference's: e at its float32 q (for very elongated
                # gaussians q is a small difference of large terms, so the float32 and the exact q
                # differ by far more than the tolerances); the derivative is that of the exact q.
                q = q + (sq.to(q.dtype) - q).detach()
            e = torch.exp(-0.5 * q.clamp_max(CUTOFF * 4))
            w = torch.where(support, e * weight[gid], torch.zeros_like(e))
            color_sum = color_sum.index_add(0, flat, w[:, None] * color[gid])
            density = density.index_add(0, flat, w)
        start = end
    return color_sum, density


def render_batched(
    xy: torch.Tensor,
    chol: torch.Tensor,
    color: torch.Tensor,
    weight: torch.Tensor,
    height: int,
    width: int,
    with_density: bool = False,
    accumulate_dtype: torch.dtype | None = None,
    budget: int = DEFAULT_BUDGET,
):
    """(B, H, W, 3) render of stacked (B, N, .) gaussians, differentiable (renderer2d.py:72-125).

    ``accumulate_dtype=torch.float64`` evaluates the reference's float32 pairs (rectangles, q and
    so the support test and exp(-q/2) from the float32 inputs) with float64 products, derivatives
    and sums: the float32 reference's render and gradients without the rounding error of float32
    sums over many pixels.
    """
    n_views, n = xy.shape[:2]
    xy_f = xy.reshape(-1, 2)
    chol_f = chol.reshape(-1, 3)
    rects = cuda_rects(xy_f, chol_f, height, width)
    conics = chol_conics(chol_f)
    view_index = torch.arange(n_views).repeat_interleave(n)
    color_f, weight_f, support = color.reshape(-1, 3), weight.reshape(-1), None
    if accumulate_dtype is not None and accumulate_dtype != xy.dtype:
        support = (xy_f.detach(), conics.detach())
        xy_f, color_f, weight_f = xy_f.to(accumulate_dtype), color_f.to(accumulate_dtype), weight_f.to(accumulate_dtype)
        conics = chol_conics(chol_f.to(accumulate_dtype))
    img, den = accumulate(
        xy_f, conics, color_f, weight_f, rects, view_index, n_views, height, width, budget=budget,
        support_inputs=support,
    )
    img = img.reshape(n_views, height, width, 3)
    if with_density:
        return img, den.reshape(n_views, height, width)
    return img


def render(xy, chol, color, weight, height: int, width: int) -> torch.Tensor:
    """(H, W, 3) render of one gaussian set."""
    return render_batched(xy[None], chol[None], color[None], weight[None], height, width)[0]


def tile_binning(rects: np.ndarray, view_index: np.ndarray, finite: np.ndarray, n_views: int, height: int, width: int):
    """Per-tile gaussian lists for 16x16 tiles: (sorted_gids, tile_ranges (n_views*T, 2)).

    A gaussian with a non-empty rectangle is listed in every tile its rectangle touches; inside
    a tile the list is in ascending gaussian index, which is the order ``index_add`` sums a pixel
    in (renderer2d.py:228-253). Integer work, so the CUDA binning must match it exactly.
    """
    tx_n = (width + TILE - 1) // TILE
    ty_n = (height + TILE - 1) // TILE
    t_per_view = tx_n * ty_n
    x0, x1, y0, y1 = (rects[:, k].astype(np.int64) for k in range(4))
    keep = (x1 >= x0) & (y1 >= y0) & finite
    keys, vals = [], []
    for g in np.nonzero(keep)[0]:
        ty_a, ty_b = y0[g] // TILE, y1[g] // TILE
        tx_a, tx_b = x0[g] // TILE, x1[g] // TILE
        ty, tx = np.meshgrid(np.arange(ty_a, ty_b + 1), np.arange(tx_a, tx_b + 1), indexing="ij")
        k = view_index[g] * t_per_view + ty.ravel() * tx_n + tx.ravel()
        keys.append(k)
        vals.append(np.full(k.shape, g, dtype=np.int64))
    n_tiles = n_views * t_per_view
    ranges = np.zeros((n_tiles, 2), dtype=np.int64)
    if not keys:
        return np.zeros(0, dtype=np.int64), ranges
    keys = np.concatenate(keys)
    vals = np.concatenate(vals)
    order = np.argsort(keys, kind="stable")
    keys, vals = keys[order], vals[order]
    starts = np.searchsorted(keys, np.arange(n_tiles), side="left")
    ends = np.searchsorted(keys, np.arange(n_tiles), side="right")
    ranges[:, 0] = np.where(ends > starts, starts, 0)
    ranges[:, 1] = np.where(ends > starts, ends, 0)
    return vals, ranges


def tile_binning_vectorized(rects: np.ndarray, view_index: np.ndarray, finite: np.ndarray, n_views: int,
                            height: int, width: int):
    """``tile_binning`` for large scenes (millions of entries): the same (gids, ranges), built with
    whole-array numpy operations instead of a loop over gaussians (pinned to ``tile_binning`` by
    the CPU tests)."""
    tx_n = (width + TILE - 1) // TILE
    ty_n = (height + TILE - 1) // TILE
    t_per_view = tx_n * ty_n
    n_tiles = n_views * t_per_view
    x0, x1, y0, y1 = (rects[:, k].astype(np.int64) for k in range(4))
    keep = (x1 >= x0) & (y1 >= y0) & finite
    gid = np.nonzero(keep)[0]
    tx_a, ty_a = x0[gid] // TILE, y0[gid] // TILE
    ntx = x1[gid] // TILE - tx_a + 1
    cnt = ntx * (y1[gid] // TILE - ty_a + 1)
    total = int(cnt.sum())
    ranges = np.zeros((n_tiles, 2), dtype=np.int64)
    if total == 0:
        return np.zeros(0, dtype=np.int64), ranges
    owner = np.repeat(np.arange(gid.size), cnt)
    local = np.arange(total, dtype=np.int64) - np.repeat(np.cumsum(cnt) - cnt, cnt)
    tiles = (view_index[gid].astype(np.int64)[owner] * t_per_view
             + (ty_a[owner] + local // ntx[owner]) * tx_n + tx_a[owner] + local % ntx[owner])
    gids = gid[owner]
    base = int(rects.shape[0])
    key = np.sort(tiles * base + gids)  # unique keys: by tile, then ascending gaussian index
    tiles, gids = key // base, key % base
    starts = np.searchsorted(tiles, np.arange(n_tiles), side="left")
    ends = np.searchsorted(tiles, np.arange(n_tiles), side="right")
    ranges[:, 0] = np.where(ends > starts, starts, 0)
    ranges[:, 1] = np.where(ends > starts, ends, 0)
    return gids, ranges


def pair_count(rects: torch.Tensor, finite: torch.Tensor) -> int:
    """Number of (gaussian, pixel-in-rect) pairs: the work unit of the throughput metric."""
    nx = (rects[:, 1].long() - rects[:, 0].long() + 1).clamp_min(0)
    ny = (rects[:, 3].long() - rects[:, 2].long() + 1).clamp_min(0)
    return int(torch.where(finite, nx * ny, torch.zeros_like(nx)).sum())
