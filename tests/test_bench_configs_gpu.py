"""Parity at the benchmark workloads' own sizes, against the CPU oracle.

  splat_4k      3840x2160, 1,000,000 gaussians (log-normal sigma, median 3 px, tail to 64 px):
                  forward on 4,096 sampled pixels (every gaussian of the pixel's tile list);
                  per-tile gaussian lists bit-exact (its longest list, about 500, is binned by the
                  per-tile sort); the same scene plus 3,000 small gaussians crowded into one tile,
                  whose list exceeds the per-tile sort and takes the radix binning: lists
                  bit-exact and the crowded tile's pixels rendered correctly;
                  gradients of 1,024 random gaussians, the 64 largest and the 64 most elongated
                  under the N(0,1) upstream gradient of the benchmark;
                  the same 128 large / elongated gaussians alone, one per 4K view, with an
                  upstream gradient only in a band around each support boundary (9 < q < 13),
                  so that a support pixel missed by the backward's line spans or the forward's
                  reach masks moves its view's result by far more than the tolerance.
  single_large  the first 20 iterations of the 1024x768 / 50,000-gaussian fit (cosine schedule
                of the full 1,000 iterations), PSNR at every iteration;
  batched_720p  one 1280x720 view with 70,000 gaussians, 20 of 1,000 iterations;
  masked_540p   one 960x540 view with 30,000 gaussians inside its mask, L2 over the mask pixels,
                20 of 600 iterations.

Tolerances (the same as the small-size tests): renders 1e-5 relative error, gradients 1e-4
relative error per tensor, tile lists bit-exact, PSNR within 0.05 dB.
At these sizes float32 gradients are not exact to 1e-4 even in the reference: a gaussian's
gradient is a sum over up to 200,000 pixels of terms that largely cancel, and for very elongated
gaussians (aspect ratio above 150 here) the Cholesky gradient is ill-conditioned. The gradient
checks therefore compare against the oracle with float64 products and sums over the reference's
float32 pairs (rectangles, q, support test and exp(-q/2) exactly as the reference computes them
in float32): the value the float32 reference approximates. Ours must be within 1e-4 of it, or
within twice the float32 reference's own distance from it (a float32 sum in another order carries
rounding error of the same size; the distance is measured in the same test and reported in the
assertion message). In the boundary-band check the colour and weight gradients (well-conditioned
sums) are held to 1e-4 outright -- a missed support pixel moves them by a percent or more -- and
the mean and Cholesky gradients, differences of large terms over a thin band (the float32
reference's own Cholesky gradients are off by up to tens of percent there), must be no less
accurate than the float32 reference over the 128 gaussians, in the worst case and the median.
Reference: src/rtgs/image2gs/renderer2d.py:156-254 (rectangles, accumulation),
src/rtgs/image2gs/fit.py:451-554 (the fit loop).
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from conftest import rel_err
from gpu_helpers import DEV, last_binning, oracle_grads
from oracle import fit as ofit
from oracle import render2d as orender
from rtgs_b200 import _native
from rtgs_b200.image2gs import synthetic
from rtgs_b200.image2gs.engine import FitEngine, pack_mask_bits
from rtgs_b200.image2gs.fit import raw_from_gaussians
from rtgs_b200.image2gs.renderer2d import render_gaussians_2d_batched

pytestmark = pytest.mark.gpu
RENDER_TOL = 1e-5
GRAD_TOL = 1e-4
PSNR_TOL = 0.05
H4K, W4K = 2160, 3840
NAMES = ("xy", "chol", "color", "weight")


def _render_forward(arena, xy, chol, color, weight, n_views, n, h, w):
    out = torch.empty(n_views, h, w, 3, device=DEV)
    _native.check(_native.lib().rtgs2d_render_forward(
        arena, xy.data_ptr(), chol.data_ptr(), color.data_ptr(), weight.data_ptr(), n_views, n, h, w,
        out.data_ptr(), None, _native.stream_ptr(DEV)))
    return out


def _render_backward(arena, up, xy, chol, color, weight, n_views, n, h, w, after_forward):
    grads = [torch.empty_like(x) for x in (xy, chol, color, weight)]
    fn = (_native.lib().rtgs2d_render_backward_after_forward if after_forward
          else _native.lib().rtgs2d_render_backward)
    _native.check(fn(arena, up.data_ptr(), None, xy.data_ptr(), chol.data_ptr(), color.data_ptr(),
                     weight.data_ptr(), n_views, n, h, w, *(g.data_ptr() for g in grads),
                     _native.stream_ptr(DEV)))
    return grads


@pytest.fixture(scope="module")
def splat4k():
    """The 4K scene, its render, its tile binning and its gradients (one forward + backward)."""
    sc = synthetic.splat_scene(0)
    m = sc.xy.shape[0]
    args = [x.to(DEV).contiguous() for x in (sc.xy, sc.chol, sc.color, sc.weight)]
    up = synthetic.splat_upstream_grad(0, 1, H4K, W4K)
    arena = _native.arena(DEV)
    img = _render_forward(arena, *args, 1, m, H4K, W4K)
    torch.cuda.synchronize()
    gids, ranges = last_binning()
    grads = _render_backward(arena, up.to(DEV), *args, 1, m, H4K, W4K, after_forward=True)
    torch.cuda.synchronize()
    rects = orender.cuda_rects(sc.xy, sc.chol, H4K, W4K)
    return dict(sc=sc, img=img, gids=gids, ranges=ranges, grads=[g.cpu() for g in grads], up=up, rects=rects)


def _check_binning(sc, rects, gids, ranges):
    finite = np.isfinite(sc.xy.numpy()).all(1)
    ogids, oranges = orender.tile_binning_vectorized(rects.numpy(), np.zeros(rects.shape[0], np.int64), finite,
                                                     1, H4K, W4K)
    assert gids.size == ogids.size > 10_000_000
    assert np.array_equal(gids.astype(np.int64), ogids)
    assert np.array_equal(ranges.astype(np.int64), oranges)
    return int((oranges[:, 1] - oranges[:, 0]).max())


def test_splat_4k_tile_lists_bit_exact(splat4k):
    longest = _check_binning(splat4k["sc"], splat4k["rects"], splat4k["gids"], splat4k["ranges"])
    assert 300 < longest <= 2048  # the per-tile sort path


def test_splat_4k_with_a_crowded_tile_takes_the_radix_binning():
    """3,000 extra gaussians (sigma 0.4 to 1 px) inside tile (100, 60) of the 4K scene: that tile's
    list exceeds the per-tile sort, so the render bins by the global radix sort. Lists bit-exact,
    and the crowded tile's 256 pixels plus 1,024 random ones rendered within tolerance."""
    base = synthetic.splat_scene(0)
    gen = torch.Generator().manual_seed(12)
    k = 3000
    xy = torch.tensor([100 * 16.0, 60 * 16.0]) + 2.0 + 12.0 * torch.rand(k, 2, generator=gen)
    sig = 0.4 + 0.6 * torch.rand(k, 2, generator=gen, dtype=torch.float64)
    chol = synthetic._chol_from_sigmas(sig[:, 0], sig[:, 1], torch.rand(k, generator=gen, dtype=torch.float64) * 3.14)
    sc = synthetic.GaussianSet(torch.cat([base.xy, xy]), torch.cat([base.chol, chol]),
                               torch.cat([base.color, torch.rand(k, 3, generator=gen)]),
                               torch.cat([base.weight, torch.ones(k)]))
    m = sc.xy.shape[0]
    args = [x.to(DEV).contiguous() for x in (sc.xy, sc.chol, sc.color, sc.weight)]
    img = _render_forward(_native.arena(DEV), *args, 1, m, H4K, W4K)
    torch.cuda.synchronize()
    gids, ranges = last_binning()
    rects = orender.cuda_rects(sc.xy, sc.chol, H4K, W4K)
    assert _check_binning(sc, rects, gids, ranges) > 2048
    yy, xx = torch.meshgrid(torch.arange(960, 976), torch.arange(1600, 1616), indexing="ij")
    px = torch.cat([xx.reshape(-1), torch.randint(0, W4K, (1024,), generator=gen)])
    py = torch.cat([yy.reshape(-1), torch.randint(0, H4K, (1024,), generator=gen)])
    _check_pixels(img, sc, rects, gids.astype(np.int64), ranges, px, py)


def test_splat_4k_forward_on_4096_sampled_pixels(splat4k):
    gen = torch.Generator().manual_seed(4)
    px = torch.randint(0, W4K, (4096,), generator=gen)
    py = torch.randint(0, H4K, (4096,), generator=gen)
    pairs = _check_pixels(splat4k["img"], splat4k["sc"], splat4k["rects"], splat4k["gids"].astype(np.int64),
                          splat4k["ranges"], px, py)
    assert pairs > 4096 * 100  # about 250 pairs per pixel on this frame


def _check_pixels(img, sc, rects, gids, ranges, px, py):
    """Render of pixels (px, py) against the oracle sum over the gaussians of the pixel's tile
    list whose rectangle holds it; returns the number of such pairs."""
    n_pix = px.numel()
    ours = img[0, py.to(DEV), px.to(DEV)].cpu()
    # Candidates: the pixel's tile list in ascending gaussian order (pinned bit-exact against the
    # oracle binning), filtered by the support rectangle; summed in that order (index_add).
    tile = (py // 16) * ((W4K + 15) // 16) + px // 16
    start = torch.from_numpy(ranges[tile.numpy(), 0].astype(np.int64))
    lens = torch.from_numpy((ranges[tile.numpy(), 1] - ranges[tile.numpy(), 0]).astype(np.int64))
    owner = torch.repeat_interleave(torch.arange(n_pix), lens)
    pos = torch.repeat_interleave(start, lens) + torch.arange(int(lens.sum())) - torch.repeat_interleave(lens.cumsum(0) - lens, lens)
    g = torch.from_numpy(gids)[pos]
    cx, cy = px[owner], py[owner]
    inside = (rects[g, 0] <= cx) & (rects[g, 1] >= cx) & (rects[g, 2] <= cy) & (rects[g, 3] >= cy)
    g, owner, cx, cy = g[inside], owner[inside], cx[inside], cy[inside]
    conics = orender.chol_conics(sc.chol[g])
    dx = (cx.float() + 0.5) - sc.xy[g, 0]
    dy = (cy.float() + 0.5) - sc.xy[g, 1]
    q = ((dx * dx) * conics[:, 0] + ((2.0 * dx) * dy) * conics[:, 1]) + (dy * dy) * conics[:, 2]
    wv = torch.where(q < 12.0, torch.exp(-0.5 * q.clamp_max(48.0)) * sc.weight[g], torch.zeros_like(q))
    ref = torch.zeros(n_pix, 3).index_add(0, owner, wv[:, None] * sc.color[g])
    err = (ours - ref).abs().max(dim=1).values / ref.abs().max(dim=1).values.clamp_min(1e-3)
    assert float(err.max()) <= RENDER_TOL
    return int(inside.sum())


def _tails(sc, rects, k=64):
    """Indices of the k largest (support rectangle area) and k most elongated gaussians."""
    area = (rects[:, 1] - rects[:, 0] + 1).clamp_min(0) * (rects[:, 3] - rects[:, 2] + 1).clamp_min(0)
    largest = torch.topk(area.double(), k).indices
    cov = orender.chol_covariance(sc.chol.double())
    tr = cov[:, 0, 0] + cov[:, 1, 1]
    det = cov[:, 0, 0] * cov[:, 1, 1] - cov[:, 0, 1] ** 2
    disc = (tr * tr / 4 - det).clamp_min(0).sqrt()
    aspect = ((tr / 2 + disc) / (tr / 2 - disc).clamp_min(1e-12)).sqrt()
    aspect = torch.where(area > 0, aspect, torch.zeros_like(aspect))
    aspect[largest] = 0
    elongated = torch.topk(aspect, k).indices
    return largest, elongated, aspect


def test_splat_4k_gradients_of_random_largest_and_elongated_gaussians(splat4k):
    sc, rects = splat4k["sc"], splat4k["rects"]
    largest, elongated, aspect = _tails(sc, rects)
    assert float(aspect[elongated].min()) > 20.0
    gen = torch.Generator().manual_seed(6)
    rand = torch.randperm(sc.xy.shape[0], generator=gen)[:1024]
    for label, sel in (("random", rand), ("largest", largest), ("elongated", elongated)):
        sub = [x[sel][None] for x in (sc.xy, sc.chol, sc.color, sc.weight)]
        # Additive splatting: a gaussian's gradient depends only on its own parameters and the
        # upstream gradient inside its rectangle, so the subset's oracle gradients are the full
        # scene's.
        exact = oracle_grads(*sub, H4K, W4K, splat4k["up"], accumulate_dtype=torch.float64)
        ref32 = oracle_grads(*sub, H4K, W4K, splat4k["up"])
        for name, g_all, r, r32 in zip(NAMES, splat4k["grads"], exact, ref32):
            ours, ref_err = g_all[sel], rel_err(r32[0], r[0])
            err = rel_err(ours, r[0])
            assert err <= max(GRAD_TOL, 2 * ref_err), (label, name, err, ref_err)


def test_splat_4k_boundary_band_of_large_and_elongated_gaussians():
    """One gaussian per 4K view (the scene's 64 largest and 64 most elongated, at their own
    positions), upstream gradient N(0,1) only where 9 < q < 13 (float64): the gradient is then a
    sum over about a hundred to a few thousand boundary pixels, and the render of the view is
    compared over the whole rectangle."""
    sc = synthetic.splat_scene(0)
    rects = orender.cuda_rects(sc.xy, sc.chol, H4K, W4K)
    largest, elongated, _ = _tails(sc, rects)
    sel = torch.cat([largest, elongated])
    gen = torch.Generator().manual_seed(8)
    arena = _native.arena(DEV)
    chunk = 16
    all_err = {name: [] for name in NAMES}
    for c0 in range(0, sel.numel(), chunk):
        idx = sel[c0:c0 + chunk]
        v = idx.numel()
        args = [x[idx][:, None] for x in (sc.xy, sc.chol, sc.color, sc.weight)]  # (v, 1, .)
        up = torch.zeros(v, H4K, W4K, 3, device=DEV)
        bands = []
        for j in range(v):
            x0, x1, y0, y1 = (int(r) for r in rects[idx[j]])
            l11, l21, l22 = (float(c) for c in sc.chol[idx[j]].double())
            s00, s01, s11 = l11 * l11, l11 * l21, l21 * l21 + l22 * l22
            det = s00 * s11 - s01 * s01
            pyy, pxx = torch.meshgrid(torch.arange(y0, y1 + 1, dtype=torch.float64),
                                      torch.arange(x0, x1 + 1, dtype=torch.float64), indexing="ij")
            dx = pxx + 0.5 - float(sc.xy[idx[j], 0])
            dy = pyy + 0.5 - float(sc.xy[idx[j], 1])
            q = (s11 * dx * dx - 2 * s01 * dx * dy + s00 * dy * dy) / det
            band = (q > 9.0) & (q < 13.0)
            vals = torch.randn(int(band.sum()), 3, generator=gen)
            by, bx = pyy[band].long(), pxx[band].long()
            up[j, by.to(DEV), bx.to(DEV)] = vals.to(DEV)
            bands.append((by, bx, vals))
            assert band.sum() > 20
        dev_args = [a.to(DEV).contiguous() for a in args]
        img = _render_forward(arena, *dev_args, v, 1, H4K, W4K)
        grads = _render_backward(arena, up, *dev_args, v, 1, H4K, W4K, after_forward=True)
        torch.cuda.synchronize()
        for j in range(v):
            x0, x1, y0, y1 = (int(r) for r in rects[idx[j]])
            hh, ww = y1 - y0 + 1, x1 - x0 + 1
            # float64 sums over the float32 reference's pairs, and the float32 reference itself
            # (see the module docstring)
            leaves = [a[j].detach().clone().requires_grad_(True) for a in args]
            v64 = [leaf.double() for leaf in leaves]
            color_sum, _ = orender.accumulate(v64[0], orender.chol_conics(v64[1]), v64[2], v64[3],
                                              rects[idx[j]][None], torch.zeros(1, dtype=torch.int32), 1, hh, ww,
                                              origin=(x0, y0),
                                              support_inputs=(args[0][j], orender.chol_conics(args[1][j])))
            ref_img = color_sum.reshape(hh, ww, 3)
            leaves32 = [a[j].detach().clone().requires_grad_(True) for a in args]
            c32, _ = orender.accumulate(leaves32[0], orender.chol_conics(leaves32[1]), leaves32[2], leaves32[3],
                                        rects[idx[j]][None], torch.zeros(1, dtype=torch.int32), 1, hh, ww,
                                        origin=(x0, y0))
            ours_img = img[j, y0:y1 + 1, x0:x1 + 1].cpu()
            assert rel_err(ours_img, ref_img) <= RENDER_TOL, ("render", int(idx[j]))
            # nothing is drawn outside the support rectangle
            assert int(img[j].ne(0).sum()) == int(img[j, y0:y1 + 1, x0:x1 + 1].ne(0).sum())
            by, bx, vals = bands[j]
            up_win = torch.zeros(hh, ww, 3, dtype=torch.float64)
            up_win[by - y0, bx - x0] = vals.double()
            (ref_img * up_win).sum().backward()
            (c32.reshape(hh, ww, 3) * up_win.float()).sum().backward()
            for name, g, leaf, leaf32 in zip(NAMES, grads, leaves, leaves32):
                ours_g = g[j].cpu().reshape(leaf.grad.shape)
                err, ref_err = rel_err(ours_g, leaf.grad), rel_err(leaf32.grad, leaf.grad)
                if name in ("color", "weight"):
                    # sums of e * up over the band: well conditioned, so the plain tolerance holds,
                    # while one missed band pixel moves them by about 1 / sqrt(band pixels) > 1%
                    assert err <= GRAD_TOL, (name, int(idx[j]), err, ref_err)
                all_err[name].append((err, ref_err))
        del up, img
    # Mean and Cholesky gradients of a thin band of an elongated gaussian are differences of large
    # terms, so float32 sums in any order carry errors well above 1e-4 (the reference's Cholesky
    # gradient is off by up to tens of percent on these gaussians): over the 128 gaussians, ours
    # must be no less accurate than the float32 reference, in the worst case and the median.
    for name in ("xy", "chol"):
        ours_e = sorted(e for e, _ in all_err[name])
        ref_e = sorted(r for _, r in all_err[name])
        assert ours_e[-1] <= max(GRAD_TOL, ref_e[-1]), (name, ours_e[-1], ref_e[-1])
        assert ours_e[len(ours_e) // 2] <= max(GRAD_TOL, ref_e[len(ref_e) // 2]), (name, ours_e, ref_e)


def _fit_trajectory(name: str, seed: int, n_iters: int = 20):
    """PSNR after each of the first n_iters iterations of workload `name` (one view), engine and
    oracle, with the cosine schedule of the full fit."""
    wl = synthetic.WORKLOADS[name]
    h, w, n, full = wl["height"], wl["width"], wl["n_fit"], wl["iterations"]
    target = synthetic.make_target(seed, wl, render_gaussians_2d_batched, DEV)
    masked = bool(wl.get("masked"))
    if masked:
        mask = synthetic.ellipse_mask(seed, h, w)
        init = synthetic.masked_fit_init(seed, n, mask)
        counts = np.array([3.0 * float(mask.sum())])
    else:
        mask = None
        init = synthetic.fit_init(seed, n, h, w)
        counts = np.array([3.0 * h * w])
    stacked = tuple(x[None] for x in (init.xy, init.chol, init.color, init.weight))
    raw = raw_from_gaussians(*(x.to(DEV) for x in stacked), h, w)
    with FitEngine(1, n, h, w, lr=1e-2, iterations=full, log_every=1, device=DEV,
                   loss_mode=_native.LOSS_MASK_ONLY if masked else _native.LOSS_MSE) as engine:
        engine.set_targets(target[None], pack_mask_bits(mask[None].to(DEV)) if masked else None)
        engine.set_raw(raw)
        engine.run(n_iters)
        iters, sums = engine.history()
        from rtgs_b200.image2gs.engine import psnr_values

        ours = [psnr_values(sums[r, :, 1], counts)[0] for r in range(len(iters))]
    _, hist = ofit.fit_views(target.cpu()[None], stacked, n_iters, lr=1e-2, log_every=1,
                             masks=None if mask is None else mask[None], t_max=full)
    ref = [v for _, v in hist[0]["psnr"]]
    assert list(iters) == list(range(n_iters))
    return np.array(ours), np.array(ref)


@pytest.mark.parametrize("name,seed", [("single_large", 1000), ("batched_720p", 1000), ("masked_540p", 1000)])
def test_first_20_iterations_of_benchmark_fits_match_oracle(name, seed):
    ours, ref = _fit_trajectory(name, seed)
    assert ours.shape == ref.shape == (20,)
    assert np.abs(ours - ref).max() <= PSNR_TOL, (name, np.abs(ours - ref).max())
    assert ref[-1] > ref[0]  # the fit makes progress over these iterations
