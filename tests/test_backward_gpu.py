"""GPU parity of gradients (renderer autograd path and the reference ABI).

Tolerance (written here, checked per tensor): max |ours - ref| / max |ref| <= 1e-4, and the
reference's own CUDA-parity bound allclose(atol=3e-4, rtol=3e-4)
(tests/test_renderer2d_cuda.py:74-87 in the reference).
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from conftest import load_golden, rel_err, t
from gpu_helpers import DEV, cuda, oracle_grads, stacked
from oracle import render2d as orender
from rtgs_b200 import _native
from rtgs_b200.core.gaussians2d import Gaussians2D
from rtgs_b200.image2gs.cuda_backend import render_batched_cuda_with_density
from rtgs_b200.image2gs.renderer2d import render_gaussian_coverage_2d, render_gaussians_2d_batched

pytestmark = pytest.mark.gpu
GRAD_TOL = 1e-4
NAMES = ("xy", "chol", "color", "weight")


def _ours(args, h, w, weight_fn):
    leaves = [a.to(DEV).clone().requires_grad_(True) for a in args]
    img = render_gaussians_2d_batched(*leaves, h, w, renderer="cuda")
    weight_fn(img).backward()
    return [leaf.grad.cpu() for leaf in leaves]


def test_gradients_match_reference_golden():
    g = load_golden("render_bwd")
    args = [t(g[f"in_{n}"]) for n in NAMES]
    grads = _ours(args, 20, 16, lambda im: (im * torch.linspace(0.5, 1.5, im.numel(), device=DEV).view_as(im)).sum())
    for n, ours in zip(NAMES, grads):
        ref = t(g[f"grad_{n}"])
        assert rel_err(ours, ref) <= GRAD_TOL, n
        assert torch.allclose(ours, ref, atol=3e-4, rtol=3e-4), n
    args2 = [t(g[f"in2_{n}"]) for n in NAMES]
    grads2 = _ours(args2, 33, 47, lambda im: im.square().sum())
    for n, ours in zip(NAMES, grads2):
        assert rel_err(ours, t(g[f"grad2_{n}"])) <= GRAD_TOL, n


def test_coverage_gradients_match_reference_golden():
    g = load_golden("render_bwd")
    leaves = [t(g[f"in3_{n}"])[0].to(DEV).clone().requires_grad_(True) for n in NAMES]
    cov = render_gaussian_coverage_2d(Gaussians2D(*leaves), 24, 28)
    (cov * torch.linspace(-1.0, 2.0, cov.numel(), device=DEV).view_as(cov)).sum().backward()
    for n, leaf in zip(NAMES, leaves):
        if n == "color":
            assert not leaf.grad.any()
            continue
        assert rel_err(leaf.grad, t(g[f"grad3_{n}"])[0]) <= GRAD_TOL, n


@pytest.mark.parametrize("seed,views,n,h,w,hi", [(0, 2, 48, 20, 16, 3.5), (1, 3, 400, 45, 61, 8.0),
                                                  (2, 1, 3000, 128, 96, 5.0), (3, 2, 60, 200, 150, 40.0)])
def test_gradients_match_oracle_random(seed, views, n, h, w, hi):
    args = stacked(seed, views, n, h, w, margin=8.0, hi=hi, off=1.0)
    gen = torch.Generator().manual_seed(100 + seed)
    up = torch.randn(views, h, w, 3, generator=gen)
    ours = _ours(args, h, w, lambda im: (im * up.to(DEV)).sum())
    ref = oracle_grads(*args, h, w, up)
    for name, a, b in zip(NAMES, ours, ref):
        assert rel_err(a, b) <= GRAD_TOL, name


def test_density_and_color_upstream_together():
    args = stacked(5, 2, 300, 40, 44, hi=6.0)
    gen = torch.Generator().manual_seed(5)
    up = torch.randn(2, 40, 44, 3, generator=gen)
    up_d = torch.randn(2, 40, 44, generator=gen)
    leaves = [a.to(DEV).clone().requires_grad_(True) for a in args]
    img, den = render_batched_cuda_with_density(*leaves, 40, 44)
    ((img * up.to(DEV)).sum() + (den * up_d.to(DEV)).sum()).backward()
    ref = oracle_grads(*args, 40, 44, up, up_d)
    for name, leaf, b in zip(NAMES, leaves, ref):
        assert rel_err(leaf.grad, b) <= GRAD_TOL, name


def test_only_requested_gradients_are_returned():
    xy, chol, color, weight = cuda(*stacked(6, 1, 30, 16, 16))
    color = color.clone().requires_grad_(True)
    render_gaussians_2d_batched(xy, chol, color, weight, 16, 16).sum().backward()
    assert color.grad is not None and torch.isfinite(color.grad).all()


def test_gradients_are_bitwise_deterministic():
    args = stacked(8, 2, 2500, 96, 80, hi=7.0)
    up = torch.randn(2, 96, 80, 3, generator=torch.Generator().manual_seed(1)).to(DEV)
    g1 = _ours(args, 96, 80, lambda im: (im * up).sum())
    g2 = _ours(args, 96, 80, lambda im: (im * up).sum())
    for a, b in zip(g1, g2):
        assert torch.equal(a, b)


def _ref_abi_inputs(seed, views, n, h, w):
    xy, chol, color, weight = stacked(seed, views, n, h, w, margin=6.0, hi=6.0, off=1.0)
    xy_f, chol_f = xy.reshape(-1, 2), chol.reshape(-1, 3)
    conics = orender.chol_conics(chol_f)
    rects = orender.cuda_rects(xy_f, chol_f, h, w)
    view = torch.arange(views, dtype=torch.int32).repeat_interleave(n)
    return xy_f, conics, color.reshape(-1, 3), weight.reshape(-1), rects, view


def test_reference_abi_forward_and_backward_match_oracle():
    views, n, h, w = 2, 500, 41, 59
    xy, conics, colors, weights, rects, view = _ref_abi_inputs(12, views, n, h, w)
    d = cuda(xy, conics, colors, weights, rects, view)
    lib = _native.lib()
    arena = _native.arena(DEV)
    out = torch.empty(views, h, w, 3, device=DEV)
    den = torch.empty(views, h, w, device=DEV)
    _native.check(lib.rtgs2d_forward(arena, *(x.data_ptr() for x in d), views * n, views, h, w, 12.0,
                                     out.data_ptr(), den.data_ptr(), None))
    leaves = [x.clone().requires_grad_(True) for x in (xy, conics, colors, weights)]
    rimg, rden = orender.accumulate(leaves[0], leaves[1], leaves[2], leaves[3], rects, view, views, h, w)
    assert rel_err(out, rimg.reshape(views, h, w, 3)) <= 1e-5
    assert rel_err(den, rden.reshape(views, h, w)) <= 1e-5
    gen = torch.Generator().manual_seed(3)
    up = torch.randn(views, h, w, 3, generator=gen)
    up_d = torch.randn(views, h, w, generator=gen)
    ((rimg * up.reshape(-1, 3)).sum() + (rden * up_d.reshape(-1)).sum()).backward()
    grads = [torch.empty_like(x) for x in (d[0], d[1], d[2], d[3])]
    up_dev, up_d_dev = up.to(DEV), up_d.to(DEV)  # keep alive until the kernels have run
    _native.check(lib.rtgs2d_backward(arena, up_dev.data_ptr(), up_d_dev.data_ptr(),
                                      *(x.data_ptr() for x in d), views * n, views, h, w, 12.0,
                                      *(g.data_ptr() for g in grads), None))
    torch.cuda.synchronize()
    for name, ours, leaf in zip(("xy", "conics", "colors", "weights"), grads, leaves):
        assert rel_err(ours, leaf.grad) <= GRAD_TOL, name



def test_reference_abi_with_conics_that_are_not_positive_definite():
    """The reference ABI takes any conic. The renderer's reach masks (forward) and line spans
    (backward) only narrow the walk for positive definite conics; indefinite, degenerate, negative
    and NaN-free extreme conics must walk their whole rectangles, exactly like the oracle."""
    h, w = 48, 64
    gen = torch.Generator().manual_seed(21)
    conics = torch.tensor([
        [0.05, 0.0, 0.02],      # positive definite, wide
        [0.5, 0.0, -0.02],      # indefinite: q < cutoff on a hyperbolic band
        [0.0, 0.0, 0.08],       # degenerate: no x dependence
        [-0.01, 0.0, 0.3],      # negative along x
        [0.1, 0.2, 0.1],        # det < 0
        [0.2, 0.09, 0.05],      # positive definite, strongly correlated
        [0.0, 0.0, 0.0],        # zero: every rectangle pixel has q = 0
        [1e-8, 0.0, 1e-8],      # nearly zero
    ], dtype=torch.float32)
    m = conics.shape[0]
    xy = torch.rand(m, 2, generator=gen) * torch.tensor([w - 20.0, h - 20.0]) + 10.0
    x0 = (xy[:, 0] - 9).floor().clamp(0, w - 1).int()
    y0 = (xy[:, 1] - 7).floor().clamp(0, h - 1).int()
    rects = torch.stack([x0, (x0 + 18).clamp(max=w - 1), y0, (y0 + 14).clamp(max=h - 1)], dim=1).int()
    colors = torch.rand(m, 3, generator=gen)
    weights = 0.2 + 0.8 * torch.rand(m, generator=gen)
    view = torch.zeros(m, dtype=torch.int32)
    d = cuda(xy, conics, colors, weights, rects, view)
    lib = _native.lib()
    arena = _native.arena(DEV)
    out = torch.empty(1, h, w, 3, device=DEV)
    den = torch.empty(1, h, w, device=DEV)
    _native.check(lib.rtgs2d_forward(arena, *(x.data_ptr() for x in d), m, 1, h, w, 12.0,
                                     out.data_ptr(), den.data_ptr(), None))
    leaves = [x.clone().requires_grad_(True) for x in (xy, conics, colors, weights)]
    rimg, rden = orender.accumulate(leaves[0], leaves[1], leaves[2], leaves[3], rects, view, 1, h, w)
    assert rel_err(out, rimg.reshape(1, h, w, 3)) <= 1e-5
    assert rel_err(den, rden.reshape(1, h, w)) <= 1e-5
    up = torch.randn(1, h, w, 3, generator=gen)
    up_d = torch.randn(1, h, w, generator=gen)
    ((rimg * up.reshape(-1, 3)).sum() + (rden * up_d.reshape(-1)).sum()).backward()
    grads = [torch.empty_like(x) for x in (d[0], d[1], d[2], d[3])]
    up_dev, up_d_dev = up.to(DEV), up_d.to(DEV)
    _native.check(lib.rtgs2d_backward(arena, up_dev.data_ptr(), up_d_dev.data_ptr(),
                                      *(x.data_ptr() for x in d), m, 1, h, w, 12.0,
                                      *(g.data_ptr() for g in grads), None))
    torch.cuda.synchronize()
    for name, ours, leaf in zip(("xy", "conics", "colors", "weights"), grads, leaves):
        for i in range(m):  # per gaussian: each one's gradient is its own rectangle's sum
            assert rel_err(ours[i], leaf.grad[i]) <= GRAD_TOL, (name, i)


def test_reference_abi_rejects_bad_arguments():
    lib = _native.lib()
    arena = _native.arena(DEV)
    out = torch.empty(1, 4, 4, 3, device=DEV)
    rc = lib.rtgs2d_forward(arena, None, None, None, None, None, None, 3, 1, 4, 4, 12.0, out.data_ptr(), None, None)
    assert rc == -1 and b"NULL" in lib.rtgs2d_last_error()
    rc = lib.rtgs2d_forward(arena, None, None, None, None, None, None, 0, 0, 4, 4, 12.0, out.data_ptr(), None, None)
    assert rc == -1
    e = ctypes.c_int64()
    assert lib.rtgs2d_arena_last_stats(arena, ctypes.byref(e), None) == 0


def test_backward_after_forward_reuses_binning_only_when_valid():
    """rtgs2d_render_backward_after_forward equals rtgs2d_render_backward bit for bit, both when it
    reuses the forward's binning and when another binning intervened (it then recomputes)."""
    from rtgs_b200 import _native

    xy, chol, color, weight = cuda(*stacked(12, 2, 300, 48, 40))
    other = cuda(*stacked(13, 2, 200, 48, 40))
    up = torch.randn(2, 48, 40, 3, generator=torch.Generator().manual_seed(3)).to(DEV)
    lib, dev = _native.lib(), xy.device
    arena, st = _native.arena(dev), _native.stream_ptr(dev)
    n = xy.shape[1]

    def fwd(args):
        out = torch.empty(2, 48, 40, 3, device=DEV)
        _native.check(lib.rtgs2d_render_forward(arena, *(t.data_ptr() for t in args), 2, args[0].shape[1], 48, 40,
                                                out.data_ptr(), None, st))

    def bwd(fn):
        grads = [torch.empty_like(t) for t in (xy, chol, color, weight)]
        _native.check(fn(arena, up.data_ptr(), None, xy.data_ptr(), chol.data_ptr(), color.data_ptr(),
                         weight.data_ptr(), 2, n, 48, 40, *(g.data_ptr() for g in grads), st))
        torch.cuda.synchronize()
        return grads

    ref = bwd(lib.rtgs2d_render_backward)
    fwd((xy, chol, color, weight))
    reused = bwd(lib.rtgs2d_render_backward_after_forward)
    fwd((xy, chol, color, weight))
    fwd(other)  # another binning in between: must recompute
    recomputed = bwd(lib.rtgs2d_render_backward_after_forward)
    for a, b, c in zip(ref, reused, recomputed):
        assert torch.equal(a, b) and torch.equal(a, c)


def test_backward_line_spans_keep_every_support_pixel():
    """Elongated, rotated, large gaussians (one per view) with the upstream gradient non-zero only
    in a band around each support boundary (9 < q < 13): the renderer backward walks only the
    ellipse's line spans and the forward only the records whose ellipse reaches a lane, and a
    support pixel missed at the boundary would move the render (per view) or the colour gradient
    (a sum over about a hundred band pixels) by far more than the tolerance."""
    from rtgs_b200.image2gs.synthetic import _chol_from_sigmas

    views, h, w = 16, 160, 160
    gen = torch.Generator().manual_seed(11)
    s1 = torch.exp(torch.rand(views, generator=gen, dtype=torch.float64) * (torch.log(torch.tensor(40.0)) - 0.7) + 0.7)
    aspect = torch.exp(torch.rand(views, generator=gen, dtype=torch.float64) * torch.log(torch.tensor(60.0)))
    theta = torch.rand(views, generator=gen, dtype=torch.float64) * torch.pi
    chol = _chol_from_sigmas(s1, (s1 / aspect).clamp(min=0.8), theta).reshape(views, 1, 3)
    xy = (torch.rand(views, 1, 2, generator=gen) * 100 + 30).float()
    color = torch.rand(views, 1, 3, generator=gen)
    weight = 0.2 + 0.8 * torch.rand(views, 1, generator=gen)
    # q of every pixel centre in float64, band 9 < q < 13 per view
    l11, l21, l22 = (chol[:, 0, k].double() for k in range(3))
    s00, s01, s11 = l11 * l11, l11 * l21, l21 * l21 + l22 * l22
    det = s00 * s11 - s01 * s01
    i00, i01, i11 = s11 / det, -s01 / det, s00 / det
    px = torch.arange(w, dtype=torch.float64) + 0.5
    py = torch.arange(h, dtype=torch.float64) + 0.5
    dx = px[None, None, :] - xy[:, 0, 0].double()[:, None, None]
    dy = py[None, :, None] - xy[:, 0, 1].double()[:, None, None]
    q = i00[:, None, None] * dx * dx + 2 * i01[:, None, None] * dx * dy + i11[:, None, None] * dy * dy
    band = ((q > 9.0) & (q < 13.0)).float()
    up = (torch.randn(views, h, w, 3, generator=gen) * band[..., None]).float()
    assert band.sum(dim=(1, 2)).min() > 20
    args = (xy, chol, color, weight)
    # The renderer forward skips records whose ellipse cannot reach a lane's pixels: a support
    # pixel skipped there would change its view's render by ~exp(-6) of the view's peak.
    img = render_gaussians_2d_batched(*cuda(*args), h, w, renderer="cuda").cpu()
    ref_img = orender.render_batched(*args, h, w)
    for v in range(views):
        assert rel_err(img[v], ref_img[v]) <= 1e-5, ("render", v)
    ours = _ours(args, h, w, lambda im: (im * up.to(DEV)).sum())
    ref = oracle_grads(*args, h, w, up)
    for name, a, b in zip(NAMES, ours, ref):
        for v in range(views):  # per view: each view's gradient is one gaussian's band sum
            assert rel_err(a[v], b[v]) <= GRAD_TOL, (name, v)
        assert torch.allclose(a, b, atol=3e-4, rtol=3e-4), name
