"""Seeded synthetic workloads for the Stage-1 benchmarks and tests.

No public dataset is involved: every target image is the accumulated render of random
anisotropic source gaussians (weight 1) plus Gaussian noise, clipped to [0, 1]; every fit starts
from a random initialisation. All random numbers come from CPU ``torch.Generator``s seeded from
the workload seed, so the parameters are identical on every machine; only the final render of a
target uses a device (pass any ``render_fn`` with the renderer2d batched signature).

Workloads (sizes from the benchmark definitions):
  single_small   128x128, 500 sources (sigma log-U[1,12]), noise sd 0.01; fit 2,000, 200 it.
  single_large   1024x768, 5,000 sources (sigma log-U[1,12]), noise sd 0.01; fit 50,000, 1,000 it.
  batched_720p   64 x 1280x720, 8,000 sources each (sigma log-U[0.5,40]), noise 0.005 N(0,1);
                 fit 70,000 per image, 1,000 it; image i uses seed base + i.
  splat_4k       3840x2160 fixed 1,000,000 gaussians, log sigma ~ N(ln 3, s^2) with
                 s = ln(64/3)/3.09 clipped to [0.35, 64], random rotation, colours U[0,1], weight 1;
                 upstream gradient N(0,1) per pixel channel.
  masked_540p    256 x 960x540 targets as batched_720p plus a binary mask: union of 3-8 random
                 ellipses covering 30-70% of the frame; fit 30,000 per view inside the mask, 600 it.
Fit initialisation: means U[0, W-1e-3) x U[0, H-1e-3), l11 and l22 log-U[0.5, 8],
l21 ~ 0.2 N(0,1), colours U[0,1], weight 0.5.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

WORKLOADS = {
    "single_small": dict(height=128, width=128, n_sources=500, sigma=(1.0, 12.0), noise=0.01,
                         n_fit=2_000, iterations=200, n_views=1),
    "single_large": dict(height=768, width=1024, n_sources=5_000, sigma=(1.0, 12.0), noise=0.01,
                         n_fit=50_000, iterations=1_000, n_views=1),
    "batched_720p": dict(height=720, width=1280, n_sources=8_000, sigma=(0.5, 40.0), noise=0.005,
                         n_fit=70_000, iterations=1_000, n_views=64),
    "masked_540p": dict(height=540, width=960, n_sources=8_000, sigma=(0.5, 40.0), noise=0.005,
                        n_fit=30_000, iterations=600, n_views=256, masked=True),
}


@dataclass
class GaussianSet:
    xy: torch.Tensor
    chol: torch.Tensor
    color: torch.Tensor
    weight: torch.Tensor

    def to(self, device) -> GaussianSet:
        return GaussianSet(self.xy.to(device), self.chol.to(device), self.color.to(device), self.weight.to(device))


def _log_uniform(gen: torch.Generator, n: int, lo: float, hi: float) -> torch.Tensor:
    u = torch.rand(n, generator=gen, dtype=torch.float64)
    return torch.exp(u * (math.log(hi) - math.log(lo)) + math.log(lo))


def _chol_from_sigmas(s1: torch.Tensor, s2: torch.Tensor, theta: torch.Tensor) -> torch.Tensor:
    """Packed Cholesky (l11, l21, l22) of R diag(s1^2, s2^2) R^T (float64 -> float32)."""
    c, s = torch.cos(theta), torch.sin(theta)
    a, b = s1 * s1, s2 * s2
    s00 = c * c * a + s * s * b
    s01 = c * s * (a - b)
    s11 = s * s * a + c * c * b
    l11 = torch.sqrt(s00)
    l21 = s01 / l11
    l22 = torch.sqrt(torch.clamp(s11 - l21 * l21, min=1e-12))
    return torch.stack([l11, l21, l22], dim=-1).float()


def source_gaussians(seed: int, k: int, height: int, width: int, sigma: tuple[float, float]) -> GaussianSet:
    """K anisotropic source gaussians: means U over the image, sigmas log-uniform, rotation U[0, pi)."""
    gen = torch.Generator().manual_seed(int(seed))
    xy = torch.rand(k, 2, generator=gen) * torch.tensor([float(width), float(height)])
    s1 = _log_uniform(gen, k, *sigma)
    s2 = _log_uniform(gen, k, *sigma)
    theta = torch.rand(k, generator=gen, dtype=torch.float64) * math.pi
    color = torch.rand(k, 3, generator=gen)
    return GaussianSet(xy, _chol_from_sigmas(s1, s2, theta), color, torch.ones(k))


def noise(seed: int, height: int, width: int, std: float) -> torch.Tensor:
    gen = torch.Generator().manual_seed(int(seed) + 0x5EED)
    return torch.randn(height, width, 3, generator=gen) * std


def make_target(seed: int, workload: dict, render_fn, device) -> torch.Tensor:
    """(H, W, 3) target: render of the sources + noise, clipped to [0, 1], on `device`."""
    h, w = workload["height"], workload["width"]
    src = source_gaussians(seed, workload["n_sources"], h, w, workload["sigma"]).to(device)
    with torch.no_grad():
        img = render_fn(src.xy[None], src.chol[None], src.color[None], src.weight[None], h, w)[0]
    return (img + noise(seed, h, w, workload["noise"]).to(device)).clamp(0.0, 1.0)


def fit_init(seed: int, n: int, height: int, width: int) -> GaussianSet:
    """Random fit initialisation (means inside the image, l11/l22 log-U[0.5, 8], l21 0.2 N(0,1))."""
    gen = torch.Generator().manual_seed(int(seed) * 2 + 1)
    xy = torch.rand(n, 2, generator=gen) * torch.tensor([width - 1e-3, height - 1e-3])
    l11 = _log_uniform(gen, n, 0.5, 8.0).float()
    l22 = _log_uniform(gen, n, 0.5, 8.0).float()
    l21 = 0.2 * torch.randn(n, generator=gen)
    color = torch.rand(n, 3, generator=gen)
    return GaussianSet(xy, torch.stack([l11, l21, l22], dim=-1), color, torch.full((n,), 0.5))


def masked_fit_init(seed: int, n: int, mask: torch.Tensor) -> GaussianSet:
    """Fit initialisation with means drawn uniformly inside the mask pixels."""
    h, w = mask.shape
    g = fit_init(seed, n, h, w)
    gen = torch.Generator().manual_seed(int(seed) * 2 + 2)
    idx = torch.nonzero(mask.reshape(-1).cpu() > 0.5).flatten()
    pick = idx[torch.randint(0, idx.numel(), (n,), generator=gen)]
    jitter = torch.rand(n, 2, generator=gen)
    g.xy = torch.stack([(pick % w).float() + jitter[:, 0] * 0.999, (pick // w).float() + jitter[:, 1] * 0.999], -1)
    return g


def ellipse_mask(seed: int, height: int, width: int, cover=(0.3, 0.7)) -> torch.Tensor:
    """Binary (H, W) union of 3-8 random ellipses covering a fraction in [cover] of the frame."""
    gen = torch.Generator().manual_seed(int(seed) + 0xA5A5)
    ys = torch.arange(height, dtype=torch.float32)[:, None] + 0.5
    xs = torch.arange(width, dtype=torch.float32)[None, :] + 0.5
    for _ in range(1000):
        k = int(torch.randint(3, 9, (1,), generator=gen))
        m = torch.zeros(height, width, dtype=torch.bool)
        for _ in range(k):
            cx = float(torch.rand(1, generator=gen)) * width
            cy = float(torch.rand(1, generator=gen)) * height
            ax = (0.08 + 0.25 * float(torch.rand(1, generator=gen))) * width
            ay = (0.08 + 0.25 * float(torch.rand(1, generator=gen))) * height
            th = float(torch.rand(1, generator=gen)) * math.pi
            c, s = math.cos(th), math.sin(th)
            u = (xs - cx) * c + (ys - cy) * s
            v = -(xs - cx) * s + (ys - cy) * c
            m |= (u / ax) ** 2 + (v / ay) ** 2 <= 1.0
        frac = float(m.float().mean())
        if cover[0] <= frac <= cover[1]:
            return m.float()
    raise RuntimeError("could not draw a mask with the requested coverage")


def splat_scene(seed: int = 0, n: int = 1_000_000, height: int = 2160, width: int = 3840) -> GaussianSet:
    """Fixed 4K splat micro-benchmark gaussians (log-normal sigmas, median 3 px, tail to 64 px)."""
    gen = torch.Generator().manual_seed(int(seed))
    xy = torch.rand(n, 2, generator=gen) * torch.tensor([float(width), float(height)])
    s = math.log(64.0 / 3.0) / 3.09
    s1 = torch.exp(torch.randn(n, generator=gen, dtype=torch.float64) * s + math.log(3.0)).clamp(0.35, 64.0)
    s2 = torch.exp(torch.randn(n, generator=gen, dtype=torch.float64) * s + math.log(3.0)).clamp(0.35, 64.0)
    theta = torch.rand(n, generator=gen, dtype=torch.float64) * math.pi
    color = torch.rand(n, 3, generator=gen)
    return GaussianSet(xy, _chol_from_sigmas(s1, s2, theta), color, torch.ones(n))


def splat_upstream_grad(seed: int, n_views: int, height: int, width: int) -> torch.Tensor:
    gen = torch.Generator().manual_seed(int(seed) + 0x6A)
    return torch.randn(n_views, height, width, 3, generator=gen)
