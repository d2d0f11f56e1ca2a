"""Fused Adam for CUDA float32 parameters (``rtgs2d_adam_step``).

``FusedAdam`` is a drop-in for ``torch.optim.Adam`` in a reference-style fit loop (render,
backward, optimizer step, scheduler step; src/rtgs/image2gs/fit.py:419-482): the same update,
state layout (``step``, ``exp_avg``, ``exp_avg_sq`` per parameter) and param-group keys that
schedulers read, but one kernel launch per step for all parameters instead of the per-parameter
ATen kernels. It is the update the native fit engine applies inside its Adam kernel; the engine
does not use this class. Supported: CUDA float32 parameters, no weight decay, amsgrad, maximize or
capturable; anything else raises ``ValueError``.
"""

from __future__ import annotations

import ctypes

import torch

from rtgs_b200 import _native

MAX_TENSORS = 16  # RTGS2D_ADAM_MAX_TENSORS


class FusedAdam(torch.optim.Optimizer):
    def __init__(self, params, lr: float = 1e-3, betas: tuple[float, float] = (0.9, 0.999), eps: float = 1e-8):
        if lr < 0.0:
            raise ValueError(f"Invalid learning rate: {lr}")
        if eps < 0.0:
            raise ValueError(f"Invalid epsilon value: {eps}")
        if not (0.0 <= betas[0] < 1.0 and 0.0 <= betas[1] < 1.0):
            raise ValueError(f"Invalid beta parameters: {betas}")
        super().__init__(params, dict(lr=lr, betas=tuple(betas), eps=eps))

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            beta1, beta2 = group["betas"]
            batches: dict[tuple[int, torch.device], list[tuple[torch.Tensor, torch.Tensor, dict]]] = {}
            for p in group["params"]:
                if p.grad is None:
                    continue
                if not p.is_cuda or p.dtype != torch.float32 or not p.is_contiguous():
                    raise ValueError("FusedAdam takes contiguous CUDA float32 parameters only")
                if p.grad.is_sparse:
                    raise ValueError("FusedAdam does not support sparse gradients")
                grad = p.grad if p.grad.is_contiguous() else p.grad.contiguous()
                state = self.state[p]
                if not state:  # torch.optim.Adam's state layout
                    state["step"] = torch.tensor(0.0)
                    state["exp_avg"] = torch.zeros_like(p)
                    state["exp_avg_sq"] = torch.zeros_like(p)
                state["step"] += 1
                batches.setdefault((int(state["step"].item()), p.device), []).append((p, grad, state))
            for (step, device), items in batches.items():
                for start in range(0, len(items), MAX_TENSORS):
                    self._launch(items[start:start + MAX_TENSORS], group["lr"], beta1, beta2, group["eps"], step, device)
        return loss

    @staticmethod
    def _launch(items, lr: float, beta1: float, beta2: float, eps: float, step: int, device: torch.device) -> None:
        n = len(items)
        ptrs = ctypes.c_void_p * n
        params = ptrs(*(p.data_ptr() for p, _, _ in items))
        grads = ptrs(*(g.data_ptr() for _, g, _ in items))
        exp_avgs = ptrs(*(s["exp_avg"].data_ptr() for _, _, s in items))
        exp_avg_sqs = ptrs(*(s["exp_avg_sq"].data_ptr() for _, _, s in items))
        sizes = (ctypes.c_int64 * n)(*(p.numel() for p, _, _ in items))
        with torch.cuda.device(device):
            _native.check(_native.lib().rtgs2d_adam_step(
                n, params, grads, exp_avgs, exp_avg_sqs, sizes, float(lr), float(beta1), float(beta2),
                float(eps), int(step), _native.stream_ptr(device)))
