"""Initialiser checks and raw transform on the device (rtgs2d_fit_set_initial) against the
reference's host checks: every malformed initialisation raises the reference's error and message
(src/rtgs/image2gs/fit.py:634-676 and fit.py:134-141), a pooled engine that rejected one
initialisation fits the next one exactly like a fresh engine, and the device raw transform
matches the host one (fit.py:375-380)."""

from __future__ import annotations

import pytest
import torch

from gpu_helpers import DEV
from rtgs_b200.core.gaussians2d import Gaussians2D
from rtgs_b200.image2gs.batched import fit_stacked
from rtgs_b200.image2gs.engine import FitEngine, clear_engine_pool
from rtgs_b200.image2gs.fit import FitConfig, NonFiniteRawParameterError, fit_image_from_initialization, raw_from_gaussians

pytestmark = pytest.mark.gpu
H, W, N = 24, 32, 12


def _image():
    yy, xx = torch.meshgrid(torch.linspace(0, 1, H), torch.linspace(0, 1, W), indexing="ij")
    return torch.stack([xx, yy, 0.5 * (xx + yy)], -1).to(DEV)


def _init():
    gen = torch.Generator().manual_seed(3)
    xy = torch.rand(N, 2, generator=gen) * torch.tensor([W - 1e-3, H - 1e-3])
    chol = torch.stack([0.5 + 2 * torch.rand(N, generator=gen), 0.2 * torch.randn(N, generator=gen),
                        0.5 + 2 * torch.rand(N, generator=gen)], -1)
    return Gaussians2D(xy, chol, torch.rand(N, 3, generator=gen), torch.rand(N, generator=gen)).to(DEV)


def _with(g: Gaussians2D, field: str, rows, value) -> Gaussians2D:
    out = Gaussians2D(g.xy.clone(), g.chol.clone(), g.color.clone(), g.weight.clone())
    getattr(out, field)[rows] = value
    return out


CFG = FitConfig(n_gaussians=N, iterations=8, log_every=4)


@pytest.mark.parametrize(
    "field,rows,value,message",
    [
        ("xy", [2, 5], float("nan"), "non-finite initial rows in xy: [2, 5]"),
        ("chol", [1], float("inf"), "non-finite initial rows in chol: [1]"),
        ("color", [0, 11], float("nan"), "non-finite initial rows in color: [0, 11]"),
        ("weight", [4], float("-inf"), "non-finite initial rows in weight: [4]"),
        ("xy", [3], torch.tensor([float(W), 1.0]), "initial Gaussians2D xy rows outside image bounds: [3]"),
        ("xy", [6], torch.tensor([1.0, -0.5]), "initial Gaussians2D xy rows outside image bounds: [6]"),
        ("chol", [7], torch.tensor([0.3, 0.0, 1.0]), "initial Gaussians2D Cholesky diagonal must exceed 0.3: rows [7]"),
        ("color", [8, 9], 1.5, "initial Gaussians2D color rows outside [0,1]: [8, 9]"),
        ("weight", [10], -0.01, "initial Gaussians2D weight rows outside [0,1]: [10]"),
    ],
)
def test_malformed_initialisations_raise_the_reference_errors(field, rows, value, message):
    bad = _with(_init(), field, rows, value.to(DEV) if isinstance(value, torch.Tensor) else value)
    with pytest.raises(ValueError) as err:
        fit_image_from_initialization(_image(), bad, CFG)
    assert str(err.value) == message


def test_first_failing_check_in_reference_order():
    bad = _with(_with(_init(), "weight", [1], 2.0), "xy", [0], torch.tensor([-1.0, 1.0], device=DEV))
    with pytest.raises(ValueError, match="xy rows outside image bounds: \\[0\\]"):
        fit_image_from_initialization(_image(), bad, CFG)
    bad = _with(_with(_init(), "chol", [2], 0.1), "color", [3], float("nan"))
    with pytest.raises(ValueError, match="non-finite initial rows in color: \\[3\\]"):
        fit_image_from_initialization(_image(), bad, CFG)  # finiteness before the diagonal check


def test_rejected_initialisation_leaves_the_pooled_engine_usable():
    clear_engine_pool()
    good = _init()
    fresh, h_fresh = fit_image_from_initialization(_image(), good, CFG)
    with pytest.raises(ValueError):
        fit_image_from_initialization(_image(), _with(good, "color", [0], 3.0), CFG)
    again, h_again = fit_image_from_initialization(_image(), good, CFG)  # the pooled engine
    assert torch.equal(fresh.xy, again.xy) and torch.equal(fresh.chol, again.chol)
    assert h_fresh["psnr"] == h_again["psnr"] and h_fresh["final_psnr"] == h_again["final_psnr"]


def test_batched_fit_rejects_only_non_finite_raw_parameters():
    g = _init()
    stacked = tuple(x[None] for x in (g.xy, g.chol, g.color, g.weight))
    images = _image()[None]
    out_of_range = (stacked[0], stacked[1], stacked[2] * 0 + 1.5, stacked[3])  # clamped, as the reference
    fit_stacked(images, out_of_range, CFG)
    nan_xy = (stacked[0].clone(), stacked[1], stacked[2], stacked[3])
    nan_xy[0][0, 5, 1] = float("nan")
    with pytest.raises(NonFiniteRawParameterError) as err:
        fit_stacked(images, nan_xy, CFG)
    assert err.value.parameter_name == "xy_raw" and err.value.row_indices == (0,)


def test_device_raw_transform_matches_host_transform():
    g = _init()
    with FitEngine(1, N, H, W, lr=1e-2, iterations=4, log_every=2, device=DEV) as engine:
        assert engine.set_initial(g.xy[None], g.chol[None], g.color[None], g.weight[None]) == 0
        ours = engine.raw()
    ref = raw_from_gaussians(g.xy[None], g.chol[None], g.color[None], g.weight[None], H, W)
    for name, value in ref.items():
        assert torch.allclose(ours[name], value, rtol=2e-6, atol=2e-6), name
