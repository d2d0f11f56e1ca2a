"""Mask coverage penalty (FitConfig.mask_coverage_weight, reference fit.py:457-459,566-572): the
reference's containment tests (tests/test_image2gs_mask_contain.py) on the native engine, and parity
of the penalised serial fit with the oracle (PSNR within 0.05 dB at every logged iteration, outside
coverage within 2%)."""

from __future__ import annotations

import pytest
import torch

from gpu_helpers import DEV
from oracle import fit as ofit
from oracle import render2d as orender
from rtgs_b200.core.gaussians2d import Gaussians2D
from rtgs_b200.image2gs import synthetic
from rtgs_b200.image2gs.fit import FitConfig, _fit_native_from_initialization, fit_image
from rtgs_b200.image2gs.renderer2d import render_gaussian_coverage_2d

pytestmark = pytest.mark.gpu


def _image_and_mask(h: int = 24, w: int = 24):
    gen = torch.Generator().manual_seed(0)
    image = torch.rand(h, w, 3, generator=gen)
    mask = torch.zeros(h, w)
    mask[6:18, 6:18] = 1.0  # central foreground box
    return image.to(DEV), mask.to(DEV)


def _outside_coverage(gaussians, mask, h, w) -> float:
    coverage = render_gaussian_coverage_2d(gaussians, h, w)
    return float((coverage * (1.0 - mask.clamp(0, 1))).sum())


def test_mask_coverage_weight_reduces_outside_spill():
    image, mask = _image_and_mask()
    shared = dict(n_gaussians=40, iterations=120, log_every=120)
    free, _ = fit_image(image, FitConfig(mask_coverage_weight=0.0, **shared), seed=0, mask=mask)
    contained, _ = fit_image(image, FitConfig(mask_coverage_weight=5.0, **shared), seed=0, mask=mask)
    assert _outside_coverage(contained, mask, 24, 24) < _outside_coverage(free, mask, 24, 24)


def test_mask_coverage_weight_requires_a_mask():
    image, _ = _image_and_mask()
    with pytest.raises(ValueError, match="requires a mask"):
        fit_image(image, FitConfig(mask_coverage_weight=1.0, iterations=3), seed=0)


def test_penalised_fit_matches_oracle():
    h, w, n = 40, 48, 120
    src = synthetic.source_gaussians(31, 40, h, w, (1.5, 6.0))
    target = orender.render(src.xy, src.chol, src.color, src.weight, h, w).clamp(0, 1)
    mask = torch.zeros(h, w)
    mask[8:30, 10:36] = 1.0
    init = synthetic.fit_init(31, n, h, w)
    iters, log_every, lam = 60, 10, 3.0
    (oxy, ochol, ocolor, oweight), ohist = ofit.fit_serial(
        target, (init.xy, init.chol, init.color, init.weight), iters, log_every=log_every,
        mask=mask, coverage_weight=lam)
    cfg = FitConfig(n_gaussians=n, iterations=iters, log_every=log_every, mask_coverage_weight=lam)
    g0 = Gaussians2D(*(x.to(DEV) for x in (init.xy, init.chol, init.color, init.weight)))
    ours, hist = _fit_native_from_initialization(target.to(DEV), target.to(DEV), g0, cfg, mask.to(DEV),
                                                 torch.zeros(2, device=DEV))
    assert [i for i, _ in hist["psnr"]] == [i for i, _ in ohist["psnr"]]
    for (_, a), (_, b) in zip(hist["psnr"], ohist["psnr"]):
        assert abs(a - b) <= 0.05
    ref_out = _outside_coverage(Gaussians2D(oxy, ochol, ocolor, oweight).to(DEV), mask.to(DEV), h, w)
    our_out = _outside_coverage(ours, mask.to(DEV), h, w)
    assert abs(our_out - ref_out) <= 0.02 * ref_out
