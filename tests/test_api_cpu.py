"""Host-side behaviour of the Python API that needs no GPU: validation, error messages,
reference-compatible configuration, initialiser, mask packing and synthetic workloads."""

from __future__ import annotations

import dataclasses
from dataclasses import replace

import numpy as np
import pytest
import torch

from conftest import load_golden, t
from rtgs_b200.core.gaussians2d import Gaussians2D, chol_covariance, chol_inverse_covariance
from rtgs_b200.image2gs import synthetic
from rtgs_b200.image2gs.engine import pack_mask_bits
from rtgs_b200.image2gs.fit import FitConfig, fit_image, fit_views, init_gaussians_2d
from rtgs_b200.image2gs.renderer2d import render_gaussians_2d, render_gaussians_2d_batched


def _cpu_gaussians(n: int = 4) -> Gaussians2D:
    gen = torch.Generator().manual_seed(0)
    return Gaussians2D(
        xy=torch.rand(n, 2, generator=gen) * 8.0,
        chol=torch.tensor([[1.5, 0.2, 1.0]]).repeat(n, 1),
        color=torch.rand(n, 3, generator=gen),
        weight=torch.rand(n, generator=gen),
    )


def test_cuda_backend_imports_without_cuda():
    import rtgs_b200.image2gs.cuda_backend as cuda_backend

    assert hasattr(cuda_backend, "render_batched_cuda")


@pytest.mark.parametrize("renderer", ["cuda", "torch", "auto"])
def test_cpu_tensors_are_rejected_loudly(renderer):
    with pytest.raises(RuntimeError, match="CUDA tensors"):
        render_gaussians_2d(_cpu_gaussians(), 8, 8, renderer=renderer)


def test_unknown_renderer_rejected():
    with pytest.raises(ValueError, match="renderer"):
        render_gaussians_2d(_cpu_gaussians(), 8, 8, renderer="bogus")


def test_batched_render_rejects_bad_shapes():
    with pytest.raises(ValueError, match=r"\(B, N, 2\)"):
        render_gaussians_2d_batched(torch.zeros(3, 2), torch.zeros(3, 3), torch.zeros(3, 3), torch.zeros(3), 8, 8)
    with pytest.raises(ValueError, match=r"\(B, N, 3\)"):
        render_gaussians_2d_batched(torch.zeros(1, 3, 2), torch.zeros(1, 3, 2), torch.zeros(1, 3, 3), torch.zeros(1, 3), 8, 8)
    with pytest.raises(ValueError, match=r"\(B, N\)"):
        render_gaussians_2d_batched(torch.zeros(1, 3, 2), torch.zeros(1, 3, 3), torch.zeros(1, 3, 3), torch.zeros(3), 8, 8)


def test_fit_config_mirrors_reference_fields_and_defaults():
    fields = {f.name: f.default for f in dataclasses.fields(FitConfig)}
    expected = {
        "n_gaussians": 640, "max_gaussians": 5000, "iterations": 300, "backend": "native",
        "adaptive_density": True, "growth_waves": 5, "relocate_fraction": 0.0,
        "structsplat_renderer": "auto", "native_renderer": "torch", "batch_views": False, "lr": 1e-2,
        "grad_init_mix": 0.7, "init_strategy": "gradient", "structure_sampling": "wse", "row_chunk": 64,
        "log_every": 50, "convergence_patience": 0, "convergence_tol": 0.05,
        "convergence_check_every": 25, "appearance_parameterization": "weight_color_9p",
        "freeze_geometry": False, "pool": False, "pool_capacity": None, "pool_triage_every": 50,
        "pool_prune_count": 32, "pool_spawn_count": 32, "pool_min_live": 1, "mask_coverage_weight": 0.0,
    }
    assert fields == expected


def test_fit_rejects_cpu_images_and_unsupported_modes():
    img = torch.rand(16, 16, 3)
    with pytest.raises(RuntimeError, match="CUDA tensors"):
        fit_image(img, FitConfig(n_gaussians=8, iterations=2), seed=0)
    for bad in (dict(backend="structsplat"), dict(init_strategy="structure_tensor"),
                dict(native_renderer="bogus"),
                # the reference's mask containment validation (fit.py:616-622)
                dict(mask_coverage_weight=-1.0), dict(mask_coverage_weight=1.0, batch_views=True),
                dict(mask_coverage_weight=1.0, pool=True),
                # the reference's pool validation (fit.py:600-616)
                dict(pool=True, freeze_geometry=True), dict(pool=True, pool_capacity=4),
                dict(pool=True, pool_min_live=0), dict(pool=True, pool_triage_every=-1),
                dict(pool=True, pool_prune_count=-1), dict(pool=True, pool_spawn_count=-1)):
        with pytest.raises(ValueError):
            fit_image(img, replace(FitConfig(n_gaussians=8, iterations=2), **bad), seed=0)
    with pytest.raises(ValueError, match="appearance_parameterization must be one of"):
        fit_image(img, FitConfig(n_gaussians=8, iterations=2, appearance_parameterization="rgb"), seed=0)
    cfg = FitConfig(n_gaussians=8, iterations=2)
    for steps, cb, msg in (((1,), None, "require diagnostic_callback"), ((True,), print, "integers"),
                           ((3,), print, r"lie in \[0, iterations\]"), ((-1,), print, "lie in")):
        with pytest.raises(ValueError, match=msg):  # the reference's checks (fit.py:593-599)
            fit_image(img, cfg, seed=0, diagnostic_callback=cb, diagnostic_steps=steps)
    with pytest.raises(ValueError, match="pool fitting does not support native fit diagnostics"):
        fit_image(img, replace(cfg, pool=True), seed=0, diagnostic_callback=print)
    with pytest.raises(ValueError, match="pool fitting supports only the default appearance"):
        fit_image(img, FitConfig(n_gaussians=8, iterations=2, pool=True,
                                 appearance_parameterization="unit_weight_bounded_8p"), seed=0)


def test_unit_weight_raw_transform_matches_oracle():
    from oracle import fit as ofit
    from rtgs_b200.image2gs.fit import raw_from_gaussians

    g = load_golden("fit_appearance")
    init = tuple(t(g[f"init_{n}"]) for n in ("xy", "chol", "color", "weight"))
    ours = raw_from_gaussians(*init, 32, 32, "unit_weight_bounded_8p")
    theirs = ofit.to_raw(*init, 32, 32, ofit.UNIT_WEIGHT_8P)
    assert ours.keys() == theirs.keys()
    for name in ours:
        assert torch.equal(ours[name], theirs[name]), name
    assert torch.equal(ours["amplitude_raw"], t(g["init_amplitude_raw"]))


def test_fit_views_batched_rejects_unsupported_modes():
    images = [torch.rand(32, 32, 3), torch.rand(32, 32, 3)]
    base = FitConfig(n_gaussians=16, iterations=1, batch_views=True)
    with pytest.raises(ValueError, match="masks"):
        fit_views(images, base, masks=[torch.ones(32, 32), torch.ones(32, 32)])
    with pytest.raises(ValueError, match="native"):
        fit_views(images, replace(base, backend="structsplat"))
    with pytest.raises(ValueError, match="early stopping"):
        fit_views(images, replace(base, convergence_patience=2))
    with pytest.raises(ValueError, match="equally sized"):
        fit_views([images[0], images[1][:16]], base)
    assert fit_views([], FitConfig(batch_views=True)) == ([], [])


def test_init_gaussians_matches_reference_on_cpu():
    g = load_golden("scene")
    ours = init_gaussians_2d(t(g["images"][0]), 80, 0.7, torch.Generator().manual_seed(0))
    for name in ("xy", "chol", "color", "weight"):
        assert torch.equal(getattr(ours, name), t(g[f"init_{name}"])), name


def test_container_math_matches_reference_ops():
    g = load_golden("rects")
    chol = t(g["chol"])
    assert torch.equal(chol_covariance(chol), t(g["cov"]))
    inv = chol_inverse_covariance(chol)
    assert torch.equal(torch.stack([inv[:, 0, 0], inv[:, 0, 1], inv[:, 1, 1]], -1), t(g["conics"]))


def test_mask_bits_match_numpy_little_endian_packbits():
    rng = np.random.default_rng(0)
    masks = rng.random((3, 7, 13)) > 0.4
    bits = pack_mask_bits(torch.from_numpy(masks.astype(np.float32)))
    ref = np.stack([np.packbits(m.reshape(-1), bitorder="little") for m in masks])
    assert np.array_equal(bits.numpy(), ref)


def test_synthetic_workloads_are_deterministic_and_in_range():
    a = synthetic.fit_init(3, 500, 96, 128)
    b = synthetic.fit_init(3, 500, 96, 128)
    assert torch.equal(a.xy, b.xy) and torch.equal(a.chol, b.chol)
    assert float(a.xy[:, 0].max()) < 128 and float(a.xy[:, 1].max()) < 96 and float(a.xy.min()) >= 0
    assert float(a.chol[:, 0].min()) >= 0.5 - 1e-6 and float(a.chol[:, 0].max()) <= 8.0 + 1e-5
    s = synthetic.source_gaussians(0, 400, 64, 64, (1.0, 12.0))
    cov = chol_covariance(s.chol.double())
    eig = torch.linalg.eigvalsh(cov)
    assert float(eig.min()) >= 0.9 and float(eig.max()) <= 12.0**2 * 1.01
    m = synthetic.ellipse_mask(5, 54, 96)
    assert 0.3 <= float(m.mean()) <= 0.7
    sc = synthetic.splat_scene(0, n=20_000, height=216, width=384)
    sig = torch.linalg.eigvalsh(chol_covariance(sc.chol.double())).sqrt()
    assert float(sig.min()) >= 0.34 and float(sig.max()) <= 64.5


def test_pool_row_store_without_rendering():
    """The reference's pool tests that need no renderer (tests/test_image2gs_pool.py)."""
    from rtgs_b200.image2gs.pool import GaussianPool2D

    g0 = Gaussians2D(xy=torch.rand(4, 2) * 20, chol=torch.tensor([[2.0, 0.0, 2.0]]).repeat(4, 1),
                     color=torch.rand(4, 3), weight=torch.full((4,), 0.5))
    with pytest.raises(ValueError, match="capacity"):
        GaussianPool2D(g0, torch.tensor([24.0, 24.0]), 2)
    pool = GaussianPool2D(g0, torch.tensor([24.0, 24.0]), 6)
    optimizer = torch.optim.Adam(pool.params(), lr=1e-2)
    ids = [id(p) for p in pool.params()]
    assert pool.live_count == 4 and pool.free_rows().tolist() == [4, 5]
    pool.park(torch.tensor([0]), optimizer)
    assert pool.live_count == 3 and pool.free_rows().tolist() == [0, 4, 5]
    pool.activate(pool.free_rows()[:1], Gaussians2D(g0.xy[:1], g0.chol[:1], g0.color[:1], g0.weight[:1]), optimizer)
    assert pool.live_count == 4 and pool.free_rows().tolist() == [4, 5]
    assert [id(p) for p in pool.params()] == ids
    assert FitConfig().pool is False


def test_load_gaussians2d_matches_reference_on_every_layout(tmp_path):
    """Archive adapters against the reference's load_gaussians2d (tests/golden/adapters.npz, made
    by tests/golden/make_golden.py): native archives unchanged, StructSplat and GaussianImage
    layouts (name variants, isotropic scales, opacity logits, clamped weights, filter variance,
    forced sources) converted to the same fields within float rounding."""
    from rtgs_b200.image2gs.adapters import detect_source, load_gaussians2d

    g = load_golden("adapters")
    for case in g["cases"].tolist():
        prefix = f"{case}__in__"
        fields = {k[len(prefix):]: g[k] for k in g if k.startswith(prefix)}
        path = tmp_path / f"{case}.npz"
        np.savez(path, **fields)
        ours = load_gaussians2d(path, source=str(g[f"{case}__source"]))
        if str(g[f"{case}__source"]) == "auto":
            expect = "native" if case == "native" else "structsplat" if case.startswith("structsplat") else "gaussianimage"
            assert detect_source(fields) == expect
        for name in ("xy", "chol", "color", "weight"):
            ref = t(g[f"{case}__out__{name}"])
            value = getattr(ours, name)
            assert value.dtype == torch.float32 and value.shape == ref.shape, (case, name)
            if name == "chol":
                # l22 = sqrt(s11 - l21^2) cancels for elongated gaussians: the reference's float32
                # factor carries that rounding (relative to the factor's largest entry), the
                # closed form here is evaluated in float64.
                tol = 1e-5 * ref.abs().max(dim=1).values + 1e-6
                assert ((value - ref).abs().max(dim=1).values <= tol).all(), (case, name)
            else:
                assert torch.allclose(value, ref, rtol=1e-5, atol=1e-6), (case, name, float((value - ref).abs().max()))
    np.savez(tmp_path / "missing.npz", means=np.zeros((3, 2), np.float32), colors=np.zeros((3, 3), np.float32),
             scales=np.ones((3, 2), np.float32))
    with pytest.raises(ValueError) as err:
        load_gaussians2d(tmp_path / "missing.npz")
    assert str(err.value) == str(g["missing__error"])


def test_loaded_gaussians_round_trip_through_native_npz(tmp_path):
    from rtgs_b200.image2gs.adapters import load_gaussians2d

    np.savez(tmp_path / "ss.npz", means=np.array([[3.0, 4.0]], np.float32), log_scales=np.zeros((1, 2), np.float32),
             rotations=np.zeros(1, np.float32), colors=np.array([[0.2, 0.4, 1.5]], np.float32))
    g = load_gaussians2d(tmp_path / "ss.npz")
    assert torch.allclose(g.xy, torch.tensor([[3.5, 4.5]]))
    assert torch.allclose(g.chol, torch.tensor([[1.0, 0.0, 1.0]]), atol=1e-6)
    assert torch.equal(g.color, torch.tensor([[0.2, 0.4, 1.0]])) and torch.equal(g.weight, torch.ones(1))
    g.save_npz(tmp_path / "native.npz")
    back = load_gaussians2d(tmp_path / "native.npz")
    for name in ("xy", "chol", "color", "weight"):
        assert torch.equal(getattr(back, name), getattr(g, name))


def test_crop_to_mask_matches_reference():
    """The masked fit's crop to the mask's box + margin (reference fit.py:792-807), against the
    reference's crop of the golden masked fit."""
    from rtgs_b200.image2gs.fit import _crop_to_mask

    g = load_golden("fit_masked")
    crop, crop_mask, offset = _crop_to_mask(t(g["image"]), t(g["mask"]))
    assert torch.equal(crop, t(g["crop"])) and torch.equal(crop_mask, t(g["crop_mask"]))
    assert torch.equal(offset, t(g["offset"]))
