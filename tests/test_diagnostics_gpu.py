"""GPU tests of the native fit diagnostics (reference: src/rtgs/image2gs/fit.py:96-131,423-520,
679-766; its own pins are tests/test_stage1_fit_seam.py:151-360).

Tolerances (written here): the diagnostic run's result and history are bit-identical to the plain
run (both run the same kernels; the diagnostic run one iteration per engine call); learning rates
equal torch's CosineAnnealingLR exactly; the first Adam update matches the closed form from the
snapshots (atol 2e-7, rtol 2e-5, the reference's pin); snapshot gradients match the oracle's
autograd gradients within 1e-4 of each field's largest magnitude; losses within 1e-5 relative of
the oracle's.
"""

from __future__ import annotations

import pytest
import torch

from conftest import load_golden, t
from gpu_helpers import DEV
from oracle import fit as ofit
from oracle import render2d as orender
from rtgs_b200.core.gaussians2d import Gaussians2D
from rtgs_b200.image2gs.fit import FitConfig, NativeFitDiagnostic, fit_image, fit_image_from_initialization, init_gaussians_2d

pytestmark = pytest.mark.gpu


def _tiny_case(masked: bool):
    image = torch.linspace(0.0, 1.0, 12 * 14 * 3, dtype=torch.float32).reshape(12, 14, 3)
    mask = None
    if masked:
        mask = torch.zeros(12, 14)
        mask[3:9, 5:11] = 1.0
    return image, mask


def _equal_gaussians(a: Gaussians2D, b: Gaussians2D) -> bool:
    return all(torch.equal(getattr(a, f), getattr(b, f)) for f in ("xy", "chol", "color", "weight"))


def _assert_first_adam_update(pre: NativeFitDiagnostic, post: NativeFitDiagnostic) -> None:
    beta1, beta2 = post.optimizer_defaults["betas"]
    eps = post.optimizer_defaults["eps"]
    for name in pre.optimizer_param_names:
        state = post.optimizer_state[name]
        step = int(state["step"].item())
        assert step == 1
        step_size = pre.lr_used / (1.0 - beta1**step)
        denom = state["exp_avg_sq"].sqrt() / (1.0 - beta2**step) ** 0.5 + eps
        expected = pre.raw_parameters[name] - step_size * state["exp_avg"] / denom
        assert torch.allclose(post.raw_parameters[name], expected, atol=2e-7, rtol=2e-5), name


@pytest.mark.parametrize("masked", [False, True])
def test_diagnostic_events_and_identity_with_the_plain_fit(masked):
    image, mask = _tiny_case(masked)
    image = image.to(DEV)
    mask = None if mask is None else mask.to(DEV)
    config = FitConfig(n_gaussians=7, iterations=3, lr=0.01, row_chunk=8, log_every=1)
    plain_g, plain_hist = fit_image(image, config, seed=193, mask=mask)
    snaps: list[NativeFitDiagnostic] = []
    diag_g, diag_hist = fit_image(image, config, seed=193, mask=mask, diagnostic_callback=snaps.append,
                                  diagnostic_steps=(0, 1, 3))
    assert _equal_gaussians(plain_g, diag_g)
    assert plain_hist == diag_hist
    assert [(s.event, s.step) for s in snaps] == [
        ("initial", 0), ("pre_update", 0), ("post_update", 1), ("checkpoint", 1), ("pre_update", 1),
        ("post_update", 2), ("pre_update", 2), ("post_update", 3), ("checkpoint", 3),
    ]
    initial = snaps[0]
    gen = torch.Generator(device=DEV).manual_seed(193)
    assert torch.equal(initial.initializer_rng_state_before, gen.get_state())
    assert initial.initial_gaussians is not None and initial.initial_gaussians.n == 7
    if not masked:  # the initialiser's draw, from the same seed (fit.py:253-277)
        g0 = init_gaussians_2d(image, 7, config.grad_init_mix, gen)
        assert _equal_gaussians(g0, initial.initial_gaussians)
        assert torch.equal(initial.initializer_rng_state_after, gen.get_state())
    assert all(v is None for v in initial.gradients.values())
    assert initial.optimizer_param_names == ("xy_raw", "diag_raw", "off_raw", "color_raw", "weight_raw")
    # learning rates: torch's own CosineAnnealingLR
    p = torch.zeros(1, requires_grad=True)
    opt = torch.optim.Adam([p], lr=config.lr)
    sched = torch.optim.lr_scheduler.CosineAnnealingLR(opt, T_max=config.iterations, eta_min=config.lr * 0.1)
    lrs = []
    for _ in range(config.iterations):
        lrs.append(float(opt.param_groups[0]["lr"]))
        opt.step()
        sched.step()
    pre = [s for s in snaps if s.event == "pre_update"]
    assert [s.lr_used for s in pre] == lrs
    assert snaps[2].scheduler_state.keys() == sched.state_dict().keys()
    assert snaps[2].optimizer_state["xy_raw"]["step"].item() == 1.0
    assert pre[0].optimizer_state["xy_raw"] == {}
    _assert_first_adam_update(pre[0], snaps[2])
    # post_update keeps the step's gradients; checkpoints carry a fresh render and loss
    for name in pre[0].gradients:
        assert torch.equal(pre[0].gradients[name], snaps[2].gradients[name])
    assert snaps[3].rendered is not None and snaps[2].rendered is None and snaps[2].loss is None


def test_diagnostic_gradients_and_losses_match_the_oracle():
    g = load_golden("fit_single")
    image = t(g["image"])
    h, w = image.shape[:2]
    init = Gaussians2D(*(t(g[f"init_{n}"]) for n in ("xy", "chol", "color", "weight")))
    config = FitConfig(n_gaussians=init.n, iterations=4, log_every=1)
    snaps: list[NativeFitDiagnostic] = []
    fit_image_from_initialization(image.to(DEV), init.to(DEV), config, diagnostic_callback=snaps.append)
    for snap in (s for s in snaps if s.event == "pre_update"):
        raw = {k: v.detach().cpu().clone().requires_grad_(True) for k, v in snap.raw_parameters.items()}
        rendered = orender.render(*ofit.build(raw, h, w), h, w)
        loss = torch.nn.functional.mse_loss(rendered, image)
        loss.backward()
        ref = float(loss.detach())
        assert abs(float(snap.loss) - ref) <= 1e-5 * ref, snap.step
        assert torch.allclose(snap.rendered.cpu(), rendered.detach(), atol=1e-5)
        for name, value in raw.items():
            ours = snap.gradients[name].cpu()
            scale = float(value.grad.abs().max())
            assert (ours - value.grad).abs().max() <= 1e-4 * scale + 1e-9, (snap.step, name)


def test_diagnostics_frozen_geometry_and_unit_weight():
    image, _ = _tiny_case(False)
    image = image.to(DEV)
    g0 = init_gaussians_2d(image, 6, 0.7, torch.Generator(device=DEV).manual_seed(41))
    traces = {}
    for arm in ("weight_color_9p", "unit_weight_bounded_8p"):
        snaps: list[NativeFitDiagnostic] = []
        config = FitConfig(n_gaussians=6, iterations=2, row_chunk=8, log_every=1, appearance_parameterization=arm,
                           freeze_geometry=True)
        fit_image_from_initialization(image, g0, config, diagnostic_callback=snaps.append, diagnostic_steps=(0, 1, 2))
        traces[arm] = snaps
    cur0, cand0 = traces["weight_color_9p"][0], traces["unit_weight_bounded_8p"][0]
    for name in ("xy_raw", "diag_raw", "off_raw"):
        assert torch.equal(cur0.raw_parameters[name], cand0.raw_parameters[name])
    expected_amplitude = torch.sigmoid(cur0.raw_parameters["weight_raw"])[:, None] * torch.sigmoid(cur0.raw_parameters["color_raw"])
    assert torch.allclose(cand0.gaussians.color, expected_amplitude, atol=1e-6, rtol=1e-5)
    for arm, snaps in traces.items():
        appearance = ("color_raw", "weight_raw") if arm == "weight_color_9p" else ("amplitude_raw",)
        assert snaps[0].optimizer_param_names == appearance
        for snap in snaps:
            if arm == "unit_weight_bounded_8p":
                assert torch.equal(snap.gaussians.weight, torch.ones_like(snap.gaussians.weight))
                assert "weight_raw" not in snap.optimizer_state
            for name in ("xy_raw", "diag_raw", "off_raw"):
                assert torch.equal(snap.raw_parameters[name], snaps[0].raw_parameters[name])
                assert snap.gradients[name] is None
            assert torch.equal(snap.gaussians.xy, snaps[0].gaussians.xy)
        pre = next(s for s in snaps if s.event == "pre_update" and s.step == 0)
        post = next(s for s in snaps if s.event == "post_update" and s.step == 1)
        _assert_first_adam_update(pre, post)
    # chain rule of the appearance parameters against the oracle's amplitude gradient
    for arm, snaps in traces.items():
        pre = next(s for s in snaps if s.event == "pre_update" and s.step == 1)
        gs = pre.gaussians
        amp = (gs.weight[:, None] * gs.color).cpu().requires_grad_(True)
        rendered = orender.render(gs.xy.cpu(), gs.chol.cpu(), amp, torch.ones(gs.n), 12, 14)
        grad_a = torch.autograd.grad(torch.nn.functional.mse_loss(rendered, image.cpu()), amp)[0]
        color, weight = gs.color.cpu(), gs.weight.cpu()[:, None]
        if arm == "weight_color_9p":
            expected = {"color_raw": grad_a * weight * color * (1.0 - color),
                        "weight_raw": (grad_a * weight * (1.0 - weight) * color).sum(dim=1)}
        else:
            expected = {"amplitude_raw": grad_a * color * (1.0 - color)}
        for name, exp in expected.items():
            err = (pre.gradients[name].cpu() - exp).abs().max()
            assert err <= 1e-4 * exp.abs().max() + 1e-9, (arm, name)


def test_diagnostics_with_early_stopping_and_mask_coverage():
    image, mask = _tiny_case(True)
    image, mask = image.to(DEV), mask.to(DEV)
    config = FitConfig(n_gaussians=7, iterations=12, log_every=2, convergence_patience=1,
                       convergence_check_every=2, convergence_tol=100.0, mask_coverage_weight=0.5)
    plain_g, plain_hist = fit_image(image, config, seed=5, mask=mask)
    snaps: list[NativeFitDiagnostic] = []
    diag_g, diag_hist = fit_image(image, config, seed=5, mask=mask, diagnostic_callback=snaps.append)
    assert plain_hist == diag_hist and _equal_gaussians(plain_g, diag_g)
    assert diag_hist["stopped_iter"] < config.iterations - 1
    assert snaps[-1].event == "post_update" and snaps[-1].step == diag_hist["stopped_iter"] + 1
    pre = [s for s in snaps if s.event == "pre_update"]
    assert all(s.loss is not None and float(s.loss) > 0 for s in pre)
