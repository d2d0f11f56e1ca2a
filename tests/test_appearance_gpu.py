"""GPU parity of the unit-weight appearance parameterisation (unit_weight_bounded_8p) against the
reference's recorded fits (tests/golden/fit_appearance.npz, made by tests/golden/make_golden.py
from src/rtgs/image2gs/fit.py:381-411 and batched.py:87-119) and the oracle.

Tolerances (written here): initial amplitude logits within 1e-4 (the logit of a product near the
clamp bounds amplifies one float32 rounding of the product); the first Adam update within the
closed-form pin of the default parameterisation (atol 2e-7, rtol 2e-5, on rows whose gradient is
not vanishing); PSNR at every logged iteration within 0.05 dB; weights exactly 1; a
geometry-frozen fit leaves the means and Cholesky factors bit-identical to the default
parameterisation's frozen fit (the reference's own pin, tests/test_stage1_fit_seam.py:257-350).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden, t
from gpu_helpers import DEV
from oracle import fit as ofit
from rtgs_b200.core.gaussians2d import Gaussians2D
from rtgs_b200.image2gs.batched import fit_stacked
from rtgs_b200.image2gs.engine import UNIT_WEIGHT_8P, FitEngine
from rtgs_b200.image2gs.fit import FitConfig, fit_image_from_initialization

pytestmark = pytest.mark.gpu
PSNR_TOL = 0.05


def _init(g, prefix: str = "init_"):
    return tuple(t(g[f"{prefix}{n}"]) for n in ("xy", "chol", "color", "weight"))


def test_unit_weight_initial_raw_and_first_update():
    g = load_golden("fit_appearance")
    image = t(g["image"])
    h, w = image.shape[:2]
    init = _init(g)
    engine = FitEngine(1, init[0].shape[0], h, w, lr=float(g["lr"]), iterations=int(g["iterations"]),
                       log_every=50, device=DEV, appearance=UNIT_WEIGHT_8P)
    try:
        assert engine.set_initial(*(x[None].to(DEV) for x in init)) == 0
        raw0 = {k: v[0].cpu() for k, v in engine.raw().items()}
        assert set(raw0) == {"xy_raw", "diag_raw", "off_raw", "amplitude_raw"}
        assert torch.allclose(raw0["amplitude_raw"], t(g["init_amplitude_raw"]), atol=1e-4, rtol=1e-5)
        _, _, _, weight = engine.params()
        assert torch.equal(weight, torch.ones_like(weight))
        engine.set_targets(image[None].to(DEV))
        engine.run(1)
        raw1 = {k: v[0].cpu() for k, v in engine.raw().items()}
    finally:
        engine.close()
    for name in raw1:
        grad = t(g[f"grad0_{name}"])
        ok = grad.abs() > 1e-6 * float(grad.abs().max())  # signs of vanishing gradients are noise
        expected = ofit.adam_first_step(raw0[name], grad, float(g["lr"]))
        assert torch.allclose(raw1[name][ok], expected[ok], atol=2e-7, rtol=2e-5), name
        assert torch.allclose(raw1[name][ok], t(g[f"step1_{name}"])[ok], atol=1e-4, rtol=1e-4), name


def test_unit_weight_fit_matches_reference_trajectory():
    g = load_golden("fit_appearance")
    cfg = FitConfig(n_gaussians=80, iterations=int(g["iterations"]), log_every=int(g["log_every"]),
                    lr=float(g["lr"]), appearance_parameterization=UNIT_WEIGHT_8P)
    fitted, hist = fit_image_from_initialization(t(g["image"]).to(DEV), Gaussians2D(*_init(g)).to(DEV), cfg)
    assert [i for i, _ in hist["psnr"]] == g["psnr_iters"].tolist()
    assert np.allclose([v for _, v in hist["psnr"]], g["psnr_vals"], atol=PSNR_TOL)
    assert abs(hist["final_psnr"] - float(g["final_psnr"])) < PSNR_TOL
    assert torch.equal(fitted.weight, torch.ones_like(fitted.weight))
    assert torch.allclose(fitted.xy.cpu(), t(g["out_xy"]), atol=2e-3)
    assert torch.allclose(fitted.color.cpu(), t(g["out_color"]), atol=2e-3)


def test_unit_weight_frozen_geometry_matches_default_geometry():
    g = load_golden("fit_appearance")
    image = t(g["image"]).to(DEV)
    g0 = Gaussians2D(*_init(g)).to(DEV)
    results = {}
    for arm in ("weight_color_9p", UNIT_WEIGHT_8P):
        cfg = FitConfig(n_gaussians=80, iterations=int(g["frozen_iterations"]), log_every=int(g["frozen_log_every"]),
                        appearance_parameterization=arm, freeze_geometry=True)
        results[arm] = fit_image_from_initialization(image, g0, cfg)
    (a, _), (b, hist) = results["weight_color_9p"], results[UNIT_WEIGHT_8P]
    assert torch.equal(a.xy, b.xy) and torch.equal(a.chol, b.chol)
    assert torch.equal(b.weight, torch.ones_like(b.weight))
    assert torch.allclose(b.xy.cpu(), t(g["frozen_xy"]), atol=1e-4)
    assert torch.allclose(b.color.cpu(), t(g["frozen_color"]), atol=1e-3)
    assert np.allclose([v for _, v in hist["psnr"]], g["frozen_psnr_vals"], atol=PSNR_TOL)


def test_unit_weight_batched_fit_matches_reference():
    g = load_golden("fit_appearance")
    gb = load_golden("fit_batched")
    cfg = FitConfig(n_gaussians=60, iterations=int(g["batched_iterations"]), log_every=int(g["batched_log_every"]),
                    batch_views=True, appearance_parameterization=UNIT_WEIGHT_8P)
    gs, hists = fit_stacked(t(g["images"]).to(DEV), _init(gb), cfg)
    for b in range(2):
        assert np.allclose([v for _, v in hists[b]["psnr"]], g["batched_psnr_vals"][b], atol=PSNR_TOL)
        assert abs(hists[b]["final_psnr"] - float(g["batched_final_psnr"][b])) < PSNR_TOL
        assert torch.equal(gs[b].weight, torch.ones_like(gs[b].weight))
        assert torch.allclose(gs[b].xy.cpu(), t(g["batched_out_xy"][b]), atol=2e-3)


def test_appearance_switch_requires_new_raw_parameters_and_rejects_unknown_codes():
    import ctypes

    from rtgs_b200 import _native

    g = load_golden("fit_appearance")
    image = t(g["image"])
    h, w = image.shape[:2]
    init = _init(g)
    engine = FitEngine(1, init[0].shape[0], h, w, lr=1e-2, iterations=4, log_every=50, device=DEV)
    try:
        engine.set_targets(image[None].to(DEV))
        assert engine.set_initial(*(x[None].to(DEV) for x in init)) == 0
        lib = _native.lib()
        assert lib.rtgs2d_fit_set_appearance(ctypes.c_void_p(engine._h), 7) != 0  # unknown code
        _native.check(lib.rtgs2d_fit_set_appearance(ctypes.c_void_p(engine._h), _native.APPEARANCE_UNIT_WEIGHT_8P))
        with pytest.raises(RuntimeError, match="set targets and raw parameters"):
            engine.run(1)  # the raw slots changed meaning: the engine refuses until they are set again
        assert engine.set_initial(*(x[None].to(DEV) for x in init)) == 0
        engine.run(1)
    finally:
        engine.close()
