"""Pooled (fixed-capacity, free-list) fitting: the reference's pool tests (tests/test_image2gs_pool.py)
on the sm_100a renderer, the native pooled fit against the reference's own pooled run
(tests/golden/fit_pool.npz: live count exact, PSNR within 0.05 dB at every logged iteration), and
the engine's parked-row contract (rtgs2d_fit_set_active / rtgs2d_fit_write_rows)."""

from __future__ import annotations

import pytest
import torch

from conftest import load_golden, t
from gpu_helpers import DEV
from rtgs_b200.core.gaussians2d import Gaussians2D
from rtgs_b200.image2gs.engine import FitEngine
from rtgs_b200.image2gs.fit import FitConfig, fit_image, fit_image_from_initialization, raw_from_gaussians
from rtgs_b200.image2gs.pool import GaussianPool2D
from rtgs_b200.image2gs.renderer2d import render_gaussians_2d

pytestmark = pytest.mark.gpu
PSNR_TOL = 0.05


def _smooth_image(h: int = 24, w: int = 24) -> torch.Tensor:
    yy, xx = torch.meshgrid(torch.linspace(0, 1, h), torch.linspace(0, 1, w), indexing="ij")
    return torch.stack([xx, yy, 0.5 * (xx + yy)], dim=-1).clamp(0, 1).to(DEV)


def _example_gaussians(n: int, h: int = 24, w: int = 24) -> Gaussians2D:
    gen = torch.Generator().manual_seed(0)
    xy = torch.rand(n, 2, generator=gen) * torch.tensor([w - 1e-3, h - 1e-3])
    chol = torch.zeros(n, 3)
    chol[:, 0] = 2.0 + torch.rand(n, generator=gen)
    chol[:, 2] = 2.0 + torch.rand(n, generator=gen)
    return Gaussians2D(xy=xy, chol=chol, color=torch.rand(n, 3, generator=gen),
                       weight=torch.rand(n, generator=gen).clamp(0.1, 0.9)).to(DEV)


def _pool(n: int, capacity: int) -> GaussianPool2D:
    return GaussianPool2D(_example_gaussians(n), torch.tensor([24.0, 24.0], device=DEV), capacity)


def test_parked_rows_are_omitted_exactly_additive():
    pool = _pool(8, 8)
    all_rows, parked, live = torch.arange(8), torch.tensor([1, 3, 5]), torch.tensor([0, 2, 4, 6, 7])
    r_all = render_gaussians_2d(pool._build_rows(all_rows.to(DEV)), 24, 24)
    r_live = render_gaussians_2d(pool._build_rows(live.to(DEV)), 24, 24)
    r_parked = render_gaussians_2d(pool._build_rows(parked.to(DEV)), 24, 24)
    assert torch.allclose(r_live + r_parked, r_all, atol=1e-6)
    optimizer = torch.optim.Adam(pool.params(), lr=1e-2)
    pool.park(parked.to(DEV), optimizer)
    assert torch.allclose(render_gaussians_2d(pool.build_active(), 24, 24), r_live, atol=1e-6)


def test_parked_rows_receive_zero_gradient():
    pool = _pool(8, 8)
    optimizer = torch.optim.Adam(pool.params(), lr=1e-2)
    parked = torch.tensor([1, 3, 5], device=DEV)
    pool.park(parked, optimizer)
    render_gaussians_2d(pool.build_active(), 24, 24).sum().backward()
    for param in pool.params():
        assert param.grad is not None and torch.count_nonzero(param.grad[parked]) == 0
    assert torch.count_nonzero(pool.params()[0].grad) > 0


def test_optimizer_is_not_rebuilt_and_recycled_moments_reset():
    pool = _pool(8, 8)
    optimizer = torch.optim.Adam(pool.params(), lr=1e-2)
    render_gaussians_2d(pool.build_active(), 24, 24).sum().backward()
    optimizer.step()
    before = [id(p) for p in optimizer.param_groups[0]["params"]]
    rows = torch.tensor([2, 5], device=DEV)
    pool.park(rows, optimizer)
    pool.activate(rows, _example_gaussians(2), optimizer)
    assert [id(p) for p in optimizer.param_groups[0]["params"]] == before
    for param in pool.params():
        state = optimizer.state[param]
        assert torch.count_nonzero(state["exp_avg"][rows]) == 0
        assert torch.count_nonzero(state["exp_avg_sq"][rows]) == 0


def test_pool_without_triage_matches_native_fit():
    image = _smooth_image()
    shared = dict(n_gaussians=16, iterations=40, log_every=40)
    native, native_hist = fit_image(image, FitConfig(**shared), seed=0)
    pooled, pooled_hist = fit_image(image, FitConfig(pool=True, pool_capacity=32, pool_triage_every=0, **shared), seed=0)
    assert pooled.n == native.n == 16
    # Same kernels on the same live rows: the parked spares change nothing, bit for bit.
    assert torch.equal(pooled.xy, native.xy) and torch.equal(pooled.color, native.color)
    assert pooled_hist["final_psnr"] == native_hist["final_psnr"]


def test_pooled_fit_with_triage_grows_and_improves():
    config = FitConfig(pool=True, n_gaussians=16, pool_capacity=48, iterations=120, pool_triage_every=30,
                       pool_prune_count=2, pool_spawn_count=8, log_every=20)
    gaussians, history = fit_image(_smooth_image(), config, seed=0)
    assert history["pool_capacity"] == 48 and history["live_count"] == gaussians.n
    assert 16 < gaussians.n <= 48
    for field in (gaussians.xy, gaussians.chol, gaussians.color, gaussians.weight):
        assert torch.isfinite(field).all()
    assert history["final_psnr"] > history["psnr"][0][1]


def test_pooled_fit_is_deterministic():
    config = FitConfig(pool=True, n_gaussians=16, pool_capacity=40, iterations=60, pool_triage_every=20,
                       pool_prune_count=2, pool_spawn_count=6, log_every=20)
    a, ha = fit_image(_smooth_image(), config, seed=3)
    b, hb = fit_image(_smooth_image(), config, seed=3)
    assert torch.equal(a.xy, b.xy) and torch.equal(a.chol, b.chol) and ha["psnr"] == hb["psnr"]


def test_pooled_fit_matches_reference_pooled_run():
    g = load_golden("fit_pool")
    init = Gaussians2D(*(t(g[f"init_{n}"]) for n in ("xy", "chol", "color", "weight"))).to(DEV)
    cfg = FitConfig(n_gaussians=init.n, iterations=int(g["iterations"]), log_every=int(g["log_every"]),
                    lr=float(g["lr"]), pool=True, pool_capacity=int(g["capacity"]),
                    pool_triage_every=int(g["triage_every"]), pool_prune_count=int(g["prune"]),
                    pool_spawn_count=int(g["spawn"]))
    fitted, hist = fit_image_from_initialization(t(g["image"]).to(DEV), init, cfg)
    assert hist["live_count"] == int(g["live_count"]) == fitted.n
    assert [i for i, _ in hist["psnr"]] == list(g["psnr_iters"])
    for (_, v), ref in zip(hist["psnr"], g["psnr_vals"]):
        assert abs(v - float(ref)) <= PSNR_TOL
    assert abs(hist["final_psnr"] - float(g["final_psnr"])) <= PSNR_TOL


def test_engine_parked_rows_render_as_the_live_subset():
    """rtgs2d_fit_set_active: the engine's render of a masked row set equals the renderer's render
    of the live rows alone; rtgs2d_fit_write_rows writes values and zeroes moments in place."""
    h, w, n = 32, 40, 24
    g = _example_gaussians(n, h, w)
    target = torch.zeros(h, w, 3, device=DEV)
    with FitEngine(1, n, h, w, lr=1e-2, iterations=10, log_every=5, device=DEV) as engine:
        engine.set_targets(target[None])
        engine.set_raw({k: v[None] for k, v in raw_from_gaussians(g.xy, g.chol, g.color, g.weight, h, w).items()})
        active = torch.ones(n, dtype=torch.bool, device=DEV)
        active[::3] = False
        engine.set_active(active[None])
        render, _ = engine.evaluate(want_render=True)
        xy, chol, color, weight = (x[0] for x in engine.params())
        live = active.nonzero(as_tuple=True)[0]
        ref = render_gaussians_2d(Gaussians2D(xy[live], chol[live], color[live], weight[live]), h, w)
        assert torch.allclose(render[0], ref, rtol=1e-6, atol=1e-6)
        engine.run(3)  # moments become non-zero on live rows
        before = engine.params()[0][0].clone()
        rows = torch.tensor([1, 4], device=DEV)
        new = Gaussians2D(torch.tensor([[5.5, 6.5], [20.5, 10.5]]), torch.tensor([[1.0, 0.1, 2.0], [3.0, 0.0, 1.0]]),
                          torch.tensor([[0.2, 0.3, 0.4], [0.9, 0.8, 0.7]]), torch.tensor([0.25, 0.75])).to(DEV)
        engine.write_rows(rows, raw_from_gaussians(new.xy, new.chol, new.color, new.weight, h, w))
        xy2, chol2, color2, weight2 = (x[0] for x in engine.params())
        assert torch.allclose(xy2[rows], new.xy, atol=2e-3) and torch.allclose(color2[rows], new.color, atol=2e-3)
        keep = torch.tensor([0, 2, 3], device=DEV)
        assert torch.equal(xy2[keep], before[keep])  # other rows untouched
        engine.set_active(None)
