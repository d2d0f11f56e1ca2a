"""Generate the golden fixtures in this folder by running the reference implementation.

Run from the repository root, in a container where the reference project is mounted:

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py /root/reference/src

It imports the reference's pure-PyTorch Stage-1 code (renderer, fit loop, batched fit,
initialiser), evaluates it on small seeded inputs on the CPU and writes compressed ``.npz``
files next to this script. Nothing at test time reads the reference; the tests read only these
fixtures. Each fixture stores its inputs and the reference outputs.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _save(name: str, **arrays) -> None:
    out = {}
    for key, value in arrays.items():
        if value is None:
            continue
        if isinstance(value, torch.Tensor):
            value = value.detach().cpu().numpy()
        out[key] = np.asarray(value)
    np.savez_compressed(HERE / f"{name}.npz", **out)
    print(f"wrote {name}.npz", {k: v.shape for k, v in out.items()})


def _stacked(seed: int, n_views: int, n: int, height: int, width: int, margin: float = 4.0):
    """Random stacked gaussians incl. off-image and edge-straddling centres (reference test style)."""
    gen = torch.Generator().manual_seed(seed)
    span = torch.tensor([width + 2 * margin, height + 2 * margin])
    xy = torch.rand(n_views, n, 2, generator=gen) * span - margin
    chol = torch.zeros(n_views, n, 3)
    chol[..., 0] = 0.5 + 3.0 * torch.rand(n_views, n, generator=gen)
    chol[..., 2] = 0.5 + 3.0 * torch.rand(n_views, n, generator=gen)
    chol[..., 1] = 0.5 * torch.randn(n_views, n, generator=gen)
    color = torch.rand(n_views, n, 3, generator=gen)
    weight = torch.rand(n_views, n, generator=gen)
    return xy, chol, color, weight


def main(ref_src: str) -> None:
    sys.path.insert(0, ref_src)
    from rtgs.core.gaussians2d import Gaussians2D, chol_covariance, chol_inverse_covariance
    from rtgs.data.synthetic import make_synthetic_scene
    from rtgs.image2gs.batched import fit_views_batched
    from rtgs.image2gs.fit import FitConfig, fit_image_from_initialization, init_gaussians_2d
    from rtgs.image2gs.renderer2d import (
        _support_rects,
        render_gaussian_coverage_2d,
        render_gaussians_2d,
        render_gaussians_2d_batched,
    )

    torch.manual_seed(0)

    # 1. Support rectangles and conics: wide random sweep plus hand-picked edge cases.
    gen = torch.Generator().manual_seed(11)
    m = 4096
    height, width = 37, 53
    xy = torch.rand(m, 2, generator=gen) * torch.tensor([width + 40.0, height + 40.0]) - 20.0
    chol = torch.empty(m, 3)
    chol[:, 0] = torch.exp(torch.rand(m, generator=gen) * 5.0 - 2.5)
    chol[:, 2] = torch.exp(torch.rand(m, generator=gen) * 5.0 - 2.5)
    chol[:, 1] = torch.randn(m, generator=gen) * 2.0
    # Centres exactly on pixel centres / pixel edges, and tiny / huge factors.
    xy[:64, 0] = torch.arange(64).float() * 0.5
    xy[64:128, 1] = torch.arange(64).float() * 0.5
    chol[128:160] = torch.tensor([0.05, 0.0, 0.05])
    chol[160:192] = torch.tensor([40.0, 5.0, 30.0])
    xy[192:200] = torch.tensor([[1e6, 5.0], [-1e6, 5.0], [5.0, 1e6], [5.0, -1e6],
                                [1e12, 1e12], [-0.49, -0.49], [width - 0.51, height - 0.51], [0.0, 0.0]])
    cov = chol_covariance(chol)
    x0, x1, y0, y1, nx, counts = _support_rects(xy, cov, height, width)
    inv = chol_inverse_covariance(chol)
    _save(
        "rects",
        xy=xy, chol=chol, height=height, width=width,
        x0=x0, x1=x1, y0=y0, y1=y1, counts=counts,
        cov=cov, conics=torch.stack([inv[:, 0, 0], inv[:, 0, 1], inv[:, 1, 1]], -1),
    )

    # 2. Forward renders (the reference CUDA-parity case, a larger mixed case, coverage).
    xy, chol, color, weight = _stacked(7, 2, 64, 24, 20)
    img = render_gaussians_2d_batched(xy, chol, color, weight, 24, 20, renderer="torch")
    xy2, chol2, color2, weight2 = _stacked(21, 3, 400, 45, 61, margin=8.0)
    chol2[0, :50, 0] *= 6.0
    chol2[1, :50, 2] *= 6.0
    img2 = render_gaussians_2d_batched(xy2, chol2, color2, weight2, 45, 61, renderer="torch")
    bg = torch.tensor([0.1, 0.2, 0.3])
    img2_bg = render_gaussians_2d_batched(xy2, chol2, color2, weight2, 45, 61, background=bg)
    g_single = Gaussians2D(xy2[2], chol2[2], color2[2], weight2[2])
    cover = render_gaussian_coverage_2d(g_single, 45, 61)
    _save("render_fwd", xy=xy, chol=chol, color=color, weight=weight, image=img,
          xy2=xy2, chol2=chol2, color2=color2, weight2=weight2, image2=img2,
          background=bg, image2_bg=img2_bg, coverage2=cover)

    # 3. Gradients: the reference CUDA-parity backward case and a squared-sum case.
    grads = {}
    leaves = [t.clone().requires_grad_(True) for t in _stacked(7, 2, 48, 20, 16)]
    image = render_gaussians_2d_batched(*leaves, 20, 16, renderer="torch")
    (image * torch.linspace(0.5, 1.5, image.numel()).view_as(image)).sum().backward()
    for name, leaf in zip(("xy", "chol", "color", "weight"), leaves):
        grads[f"in_{name}"] = leaf.detach()
        grads[f"grad_{name}"] = leaf.grad
    leaves2 = [t.clone().requires_grad_(True) for t in _stacked(5, 2, 200, 33, 47, margin=6.0)]
    render_gaussians_2d_batched(*leaves2, 33, 47).square().sum().backward()
    for name, leaf in zip(("xy", "chol", "color", "weight"), leaves2):
        grads[f"in2_{name}"] = leaf.detach()
        grads[f"grad2_{name}"] = leaf.grad
    # Coverage (density channel) gradient.
    leaves3 = [t.clone().requires_grad_(True) for t in _stacked(9, 1, 60, 24, 28)]
    g3 = Gaussians2D(*(t[0] for t in leaves3))
    cov3 = render_gaussian_coverage_2d(g3, 24, 28)
    (cov3 * torch.linspace(-1.0, 2.0, cov3.numel()).view_as(cov3)).sum().backward()
    for name, leaf in zip(("xy", "chol", "color", "weight"), leaves3):
        grads[f"in3_{name}"] = leaf.detach()
        grads[f"grad3_{name}"] = leaf.grad
    _save("render_bwd", **grads)

    # 4. The standard reference test scene images (8 views 32x32, first two) + initialiser.
    scene = make_synthetic_scene(n_gaussians=25, n_cameras=8, image_size=32, seed=0)
    images = torch.stack([scene.images[0], scene.images[1]])
    g_init = init_gaussians_2d(images[0], 80, 0.7, torch.Generator().manual_seed(0))
    _save("scene", images=images, init_xy=g_init.xy, init_chol=g_init.chol,
          init_color=g_init.color, init_weight=g_init.weight)

    # 5. Single-image native fit from a supplied initialisation (fit.py:309-352).
    cfg = FitConfig(n_gaussians=80, iterations=40, log_every=10, lr=1e-2)
    fitted, hist = fit_image_from_initialization(images[0], g_init, cfg)
    _save("fit_single", image=images[0], init_xy=g_init.xy, init_chol=g_init.chol,
          init_color=g_init.color, init_weight=g_init.weight,
          iterations=cfg.iterations, log_every=cfg.log_every, lr=cfg.lr,
          out_xy=fitted.xy, out_chol=fitted.chol, out_color=fitted.color, out_weight=fitted.weight,
          psnr_iters=np.array([i for i, _ in hist["psnr"]]),
          psnr_vals=np.array([v for _, v in hist["psnr"]]),
          final_psnr=hist["final_psnr"], final_psnr_full=hist["final_psnr_full"])

    # 6. Batched fit (batched.py:39-170) on the two scene views, seeds 0 and 1.
    bcfg = FitConfig(n_gaussians=60, iterations=30, log_every=10, batch_views=True)
    gs, hists = fit_views_batched([images[0], images[1]], bcfg, seed=0)
    inits = [init_gaussians_2d(images[i], 60, 0.7, torch.Generator().manual_seed(i)) for i in range(2)]
    _save("fit_batched", images=images, iterations=bcfg.iterations, log_every=bcfg.log_every,
          init_xy=torch.stack([g.xy for g in inits]), init_chol=torch.stack([g.chol for g in inits]),
          init_color=torch.stack([g.color for g in inits]), init_weight=torch.stack([g.weight for g in inits]),
          out_xy=torch.stack([g.xy for g in gs]), out_chol=torch.stack([g.chol for g in gs]),
          out_color=torch.stack([g.color for g in gs]), out_weight=torch.stack([g.weight for g in gs]),
          psnr_vals=np.array([[v for _, v in h["psnr"]] for h in hists]),
          psnr_iters=np.array([i for i, _ in hists[0]["psnr"]]),
          final_psnr=np.array([h["final_psnr"] for h in hists]))

    # 7. Single-gaussian known answers (tests/test_image2gs.py:14-39 in the reference).
    single = Gaussians2D(torch.tensor([[8.5, 8.5]]), torch.tensor([[2.0, 0.0, 2.0]]),
                         torch.tensor([[1.0, 0.5, 0.25]]), torch.tensor([1.0]))
    _save("single", image=render_gaussians_2d(single, 17, 17))


def pool_fixture(ref_src: str) -> None:
    """8. Pooled fit with triage (pool.py:210-291) from a fixed initialisation of the scene image."""
    sys.path.insert(0, ref_src)
    from rtgs.data.synthetic import make_synthetic_scene
    from rtgs.image2gs.fit import FitConfig, init_gaussians_2d
    from rtgs.image2gs.pool import fit_pooled_from_initialization

    torch.manual_seed(0)
    scene = make_synthetic_scene(n_gaussians=25, n_cameras=8, image_size=32, seed=0)
    image = scene.images[0]
    g_init = init_gaussians_2d(image, 40, 0.7, torch.Generator().manual_seed(3))
    cfg = FitConfig(n_gaussians=40, iterations=60, log_every=10, pool=True, pool_capacity=64,
                    pool_triage_every=15, pool_prune_count=3, pool_spawn_count=6)
    fitted, hist = fit_pooled_from_initialization(image, image, g_init, cfg, None, image.new_zeros(2))
    _save("fit_pool", image=image, init_xy=g_init.xy, init_chol=g_init.chol,
          init_color=g_init.color, init_weight=g_init.weight,
          iterations=cfg.iterations, log_every=cfg.log_every, lr=cfg.lr, capacity=cfg.pool_capacity,
          triage_every=cfg.pool_triage_every, prune=cfg.pool_prune_count, spawn=cfg.pool_spawn_count,
          out_xy=fitted.xy, out_chol=fitted.chol, out_color=fitted.color, out_weight=fitted.weight,
          psnr_iters=np.array([i for i, _ in hist["psnr"]]),
          psnr_vals=np.array([v for _, v in hist["psnr"]]),
          final_psnr=hist["final_psnr"], live_count=hist["live_count"])


def adapters_fixture(ref_src: str) -> None:
    """9. Archive adapters (adapters.py:13-82): one archive per layout and naming variant, written
    to a temporary folder, read by the reference's load_gaussians2d. Stored per case: the archive's
    arrays (``<case>__in__<field>``), the requested source and the four output fields."""
    import tempfile

    sys.path.insert(0, ref_src)
    from rtgs.image2gs.adapters import load_gaussians2d

    gen = np.random.default_rng(9)
    n = 50

    def angles(k=n):
        return gen.uniform(-np.pi, np.pi, k).astype(np.float32)

    cases = {
        "native": ("auto", dict(xy=gen.uniform(0, 40, (n, 2)), chol=np.stack([gen.uniform(0.4, 5, n),
                   gen.normal(0, 1, n), gen.uniform(0.4, 5, n)], -1), color=gen.uniform(0, 1, (n, 3)),
                   weight=gen.uniform(0, 1, n))),
        "structsplat": ("auto", dict(means=gen.uniform(0, 40, (n, 2)), log_scales=gen.normal(0.5, 1.0, (n, 2)),
                        rotations=angles(), colors=gen.normal(0.5, 0.6, (n, 3)), opacities=gen.normal(0, 2, n),
                        filter_variance=gen.normal(0.1, 0.2, n))),
        "structsplat_plain": ("auto", dict(means=gen.uniform(0, 40, (n, 2)), log_scales=gen.normal(0, 1.5, (n, 2)),
                              rotations=angles(), colors=gen.uniform(0, 1, (n, 3)))),
        "gi_scales_opacity": ("auto", dict(xy=gen.uniform(0, 40, (n, 2)), scales=gen.uniform(0.01, 9, (n, 2)),
                              rotation=angles()[:, None], color=gen.normal(0.5, 0.6, (n, 3)),
                              opacity=gen.normal(0.5, 0.6, (n, 1)))),
        "gi_isotropic_weight": ("auto", dict(positions=gen.uniform(0, 40, (n, 2)), scale=gen.uniform(0.2, 4, n),
                                angles=angles(), rgb=gen.uniform(0, 1, (n, 3)), weight=gen.uniform(-0.5, 1.5, n))),
        "gi_no_weight": ("auto", dict(means=gen.uniform(0, 40, (n, 2)), scaling=gen.uniform(0.3, 3, (n, 2)),
                         angle=angles(), colors=gen.uniform(0, 1, (n, 3)))),
        "forced_gaussianimage": ("gaussianimage", dict(means=gen.uniform(0, 40, (n, 2)),
                                 log_scales=gen.normal(0, 1, (n, 2)), rotations=angles(),
                                 colors=gen.uniform(0, 1, (n, 3)), opacities=gen.normal(0, 1, n),
                                 filter_variance=gen.uniform(0, 1, n))),
        "forced_structsplat_scales": ("structsplat", dict(xy=gen.uniform(0, 40, (n, 2)),
                                      scales=gen.uniform(0.5, 3, (n, 1)), rotation=angles(),
                                      color=gen.uniform(0, 1, (n, 3)), filter_variance=gen.uniform(0, 1, (n, 1)))),
    }
    out = {}
    with tempfile.TemporaryDirectory() as tmp:
        for name, (source, fields) in cases.items():
            fields = {k: np.asarray(v, dtype=np.float32) for k, v in fields.items()}
            path = Path(tmp) / f"{name}.npz"
            np.savez(path, **fields)
            g = load_gaussians2d(path, source=source)
            for k, v in fields.items():
                out[f"{name}__in__{k}"] = v
            out[f"{name}__source"] = np.array(source)
            for k in ("xy", "chol", "color", "weight"):
                out[f"{name}__out__{k}"] = getattr(g, k).numpy()
        missing = Path(tmp) / "missing.npz"
        np.savez(missing, means=np.zeros((3, 2), np.float32), colors=np.zeros((3, 3), np.float32),
                 scales=np.ones((3, 2), np.float32))
        try:
            load_gaussians2d(missing)
        except ValueError as err:
            out["missing__error"] = np.array(str(err))
    out["cases"] = np.array(list(cases))
    _save("adapters", **out)


def appearance_fixture(ref_src: str) -> None:
    """10. The unit-weight appearance (fit.py:381-411): the native fit of the scene image from a
    fixed initialisation with unit_weight_bounded_8p, its step-0 diagnostics (initial raw
    parameters, the first gradients and the first update), a geometry-frozen run and the batched
    fit (batched.py:87-119) of both scene views."""
    sys.path.insert(0, ref_src)
    from rtgs.data.synthetic import make_synthetic_scene
    from rtgs.image2gs.batched import fit_views_batched
    from rtgs.image2gs.fit import FitConfig, fit_image_from_initialization, init_gaussians_2d

    arm = "unit_weight_bounded_8p"
    scene = make_synthetic_scene(n_gaussians=25, n_cameras=8, image_size=32, seed=0)
    images = torch.stack([scene.images[0], scene.images[1]])
    g_init = init_gaussians_2d(images[0], 80, 0.7, torch.Generator().manual_seed(0))
    snaps = []
    cfg = FitConfig(n_gaussians=80, iterations=40, log_every=10, lr=1e-2, appearance_parameterization=arm)
    fitted, hist = fit_image_from_initialization(images[0], g_init, cfg, diagnostic_callback=snaps.append,
                                                 diagnostic_steps=(0, 1))
    pre = next(s for s in snaps if s.event == "pre_update" and s.step == 0)
    post = next(s for s in snaps if s.event == "post_update" and s.step == 1)
    fcfg = FitConfig(n_gaussians=80, iterations=10, log_every=5, lr=1e-2, appearance_parameterization=arm,
                     freeze_geometry=True)
    frozen, fhist = fit_image_from_initialization(images[0], g_init, fcfg)
    bcfg = FitConfig(n_gaussians=60, iterations=30, log_every=10, batch_views=True, appearance_parameterization=arm)
    gs, hists = fit_views_batched([images[0], images[1]], bcfg, seed=0)
    _save("fit_appearance", image=images[0], images=images, init_xy=g_init.xy, init_chol=g_init.chol,
          init_color=g_init.color, init_weight=g_init.weight,
          iterations=cfg.iterations, log_every=cfg.log_every, lr=cfg.lr,
          init_amplitude_raw=pre.raw_parameters["amplitude_raw"],
          grad0_xy_raw=pre.gradients["xy_raw"], grad0_diag_raw=pre.gradients["diag_raw"],
          grad0_off_raw=pre.gradients["off_raw"], grad0_amplitude_raw=pre.gradients["amplitude_raw"],
          step1_xy_raw=post.raw_parameters["xy_raw"], step1_diag_raw=post.raw_parameters["diag_raw"],
          step1_off_raw=post.raw_parameters["off_raw"], step1_amplitude_raw=post.raw_parameters["amplitude_raw"],
          out_xy=fitted.xy, out_chol=fitted.chol, out_color=fitted.color, out_weight=fitted.weight,
          psnr_iters=np.array([i for i, _ in hist["psnr"]]),
          psnr_vals=np.array([v for _, v in hist["psnr"]]),
          final_psnr=hist["final_psnr"],
          frozen_iterations=fcfg.iterations, frozen_log_every=fcfg.log_every,
          frozen_xy=frozen.xy, frozen_chol=frozen.chol, frozen_color=frozen.color, frozen_weight=frozen.weight,
          frozen_psnr_vals=np.array([v for _, v in fhist["psnr"]]), frozen_final_psnr=fhist["final_psnr"],
          batched_iterations=bcfg.iterations, batched_log_every=bcfg.log_every,
          batched_out_color=torch.stack([g.color for g in gs]), batched_out_xy=torch.stack([g.xy for g in gs]),
          batched_out_weight=torch.stack([g.weight for g in gs]),
          batched_psnr_vals=np.array([[v for _, v in h["psnr"]] for h in hists]),
          batched_final_psnr=np.array([h["final_psnr"] for h in hists]))


def masked_fixture(ref_src: str) -> None:
    """11. The masked serial fit (fit.py:309-352, 355-554): crop to the mask's box + margin
    (fit.py:792-807), target = image * mask, (0.1 + 0.9 mask)-weighted MSE (fit.py:557-563), the
    optional coverage penalty outside the mask (fit.py:566-572), final_psnr = masked_psnr against
    the unmasked crop, centres restored by the crop offset. Without and with the penalty."""
    sys.path.insert(0, ref_src)
    from rtgs.core.gaussians2d import Gaussians2D
    from rtgs.data.synthetic import make_synthetic_scene
    from rtgs.image2gs.fit import FitConfig, _crop_to_mask, fit_image_from_initialization, init_gaussians_2d

    scene = make_synthetic_scene(n_gaussians=25, n_cameras=8, image_size=32, seed=0)
    image = scene.images[0]
    mask = torch.zeros(32, 32)
    mask[8:24, 6:22] = 1.0
    mask[12:16, 20:26] = 1.0
    crop, crop_mask, offset = _crop_to_mask(image, mask)
    g_init = init_gaussians_2d(crop * crop_mask[..., None], 60, 0.7, torch.Generator().manual_seed(3))
    out = {"image": image, "mask": mask, "crop": crop, "crop_mask": crop_mask, "offset": offset,
           "init_xy": g_init.xy, "init_chol": g_init.chol, "init_color": g_init.color,
           "init_weight": g_init.weight}
    for tag, lam in (("plain", 0.0), ("penalised", 2.0)):
        cfg = FitConfig(n_gaussians=60, iterations=40, log_every=10, lr=1e-2, mask_coverage_weight=lam)
        fitted, hist = fit_image_from_initialization(image, Gaussians2D(g_init.xy.clone(), g_init.chol.clone(),
                                                                        g_init.color.clone(),
                                                                        g_init.weight.clone()), cfg, mask=mask)
        out.update({f"{tag}_weight_lambda": lam, f"{tag}_iterations": cfg.iterations,
                    f"{tag}_log_every": cfg.log_every, f"{tag}_lr": cfg.lr,
                    f"{tag}_out_xy": fitted.xy, f"{tag}_out_chol": fitted.chol,
                    f"{tag}_out_color": fitted.color, f"{tag}_out_weight": fitted.weight,
                    f"{tag}_psnr_iters": np.array([i for i, _ in hist["psnr"]]),
                    f"{tag}_psnr_vals": np.array([v for _, v in hist["psnr"]]),
                    f"{tag}_final_psnr": hist["final_psnr"], f"{tag}_final_psnr_full": hist["final_psnr_full"]})
    _save("fit_masked", **out)


if __name__ == "__main__":
    # make_golden.py [REF_SRC] [--only main|pool|adapters|appearance]
    args = [a for a in sys.argv[1:]
            if not a.startswith("--") and a not in ("main", "pool", "adapters", "appearance", "masked")]
    ref = args[0] if args else "/root/reference/src"
    only = sys.argv[sys.argv.index("--only") + 1] if "--only" in sys.argv else None
    if only in (None, "main"):
        main(ref)
    if only in (None, "pool"):
        pool_fixture(ref)
    if only in (None, "adapters"):
        adapters_fixture(ref)
    if only in (None, "appearance"):
        appearance_fixture(ref)
    if only in (None, "masked"):
        masked_fixture(ref)
