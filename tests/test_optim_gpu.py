"""GPU tests of the fused multi-tensor Adam step (rtgs2d_adam_step, rtgs_b200.image2gs.optim) against
torch.optim.Adam, the optimizer of the reference's fit loop (src/rtgs/image2gs/fit.py:419-422).

Tolerances (written here): after every step the parameters and both moments match torch's within
2e-5 of each tensor's largest magnitude (+2e-7; the reference pins the first update at rtol 2e-5,
tests/test_stage1_fit_seam.py:239-254; torch's CUDA Adam fuses the moment updates' multiply-adds,
which moves an entry that nearly cancels by an ulp of the terms, and the fused step's square root
and last division are hardware approximations); the state layout and the learning rates a cosine
schedule sets are torch's exactly.
"""

from __future__ import annotations

import pytest
import torch

from gpu_helpers import DEV
from oracle import fit as ofit
from rtgs_b200.image2gs import synthetic
from rtgs_b200.image2gs.optim import FusedAdam
from rtgs_b200.image2gs.renderer2d import render_gaussians_2d_batched

pytestmark = pytest.mark.gpu


def _close(x: torch.Tensor, ref: torch.Tensor) -> bool:
    return float((x - ref).abs().max()) <= 2e-5 * float(ref.abs().max()) + 2e-7


def _pair(shapes, seed=0):
    gen = torch.Generator().manual_seed(seed)
    base = [torch.randn(*s, generator=gen) for s in shapes]
    ours = [b.clone().to(DEV).requires_grad_(True) for b in base]
    ref = [b.clone().to(DEV).requires_grad_(True) for b in base]
    return ours, ref


def test_fused_adam_matches_torch_adam_with_a_cosine_schedule():
    shapes = [(50, 2), (50, 2), (50,), (50, 3), (50,), (7,), (1000, 3)] * 3  # 21 tensors: two launches
    ours, ref = _pair(shapes)
    opt_a = FusedAdam(ours, lr=1e-2)
    opt_b = torch.optim.Adam(ref, lr=1e-2)
    sch_a = torch.optim.lr_scheduler.CosineAnnealingLR(opt_a, T_max=30, eta_min=1e-3)
    sch_b = torch.optim.lr_scheduler.CosineAnnealingLR(opt_b, T_max=30, eta_min=1e-3)
    gen = torch.Generator().manual_seed(1)
    for it in range(30):
        for a, b in zip(ours, ref):
            g = torch.randn(a.shape, generator=gen).to(DEV) * (10.0 ** (it % 5 - 2))
            a.grad = g.clone()
            b.grad = g.clone()
        opt_a.step()
        opt_b.step()
        sch_a.step()
        sch_b.step()
        assert opt_a.param_groups[0]["lr"] == opt_b.param_groups[0]["lr"]
        for a, b in zip(ours, ref):
            sa, sb = opt_a.state[a], opt_b.state[b]
            assert float(sa["step"]) == float(sb["step"]) == it + 1
            assert _close(sa["exp_avg"], sb["exp_avg"]), it
            assert _close(sa["exp_avg_sq"], sb["exp_avg_sq"]), it
            assert _close(a.detach(), b.detach()), it
    assert set(opt_a.state[ours[0]]) == set(opt_b.state[ref[0]])


def test_fused_adam_skips_parameters_without_gradients_and_rejects_cpu():
    ours, _ = _pair([(4, 2), (4,)])
    before0, before1 = ours[0].detach().clone(), ours[1].detach().clone()
    ours[0].grad = torch.ones_like(ours[0])
    opt = FusedAdam(ours, lr=0.1)
    opt.step()
    assert torch.equal(ours[1].detach(), before1) and ours[1] not in opt.state
    # first step with a unit gradient: p - lr * 1 / (1 + eps)
    assert torch.allclose(ours[0].detach(), before0 - 0.1, rtol=0, atol=1e-6)
    cpu = torch.zeros(3, requires_grad=True)
    cpu.grad = torch.ones(3)
    with pytest.raises(ValueError, match="CUDA float32"):
        FusedAdam([cpu], lr=0.1).step()


def test_reference_style_loop_with_the_cuda_renderer_and_fused_adam():
    """The reference's loop shape (build, render, MSE, backward, step, schedule) with this package's
    autograd renderer and FusedAdam tracks the oracle's loop (torch Adam, CPU renderer)."""
    h, w, n, iters = 24, 28, 40, 12
    target = torch.rand(h, w, 3, generator=torch.Generator().manual_seed(3))
    g = synthetic.fit_init(5, n, h, w)
    init = (g.xy[None], g.chol[None], g.color[None], g.weight[None])
    _, ohist = ofit.fit_views(target[None], init, iters, lr=1e-2, log_every=1)
    raw = {k: v.detach().clone().to(DEV).requires_grad_(True) for k, v in ofit.to_raw(*init, h, w).items()}
    opt = FusedAdam(list(raw.values()), lr=1e-2)
    sched = torch.optim.lr_scheduler.CosineAnnealingLR(opt, T_max=iters, eta_min=1e-3)
    tdev = target.to(DEV)
    for it in range(iters):
        opt.zero_grad()
        xy, chol, color, weight = ofit.build(raw, h, w)
        rendered = render_gaussians_2d_batched(xy, chol, color, weight, h, w, renderer="cuda")
        loss = torch.nn.functional.mse_loss(rendered[0], tdev)
        psnr = float(-10.0 * torch.log10(torch.nn.functional.mse_loss(rendered[0].detach().clamp(0, 1), tdev)))
        assert abs(psnr - ohist[0]["psnr"][it][1]) < 0.05, it
        loss.backward()
        opt.step()
        sched.step()
