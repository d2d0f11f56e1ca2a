"""Container for a set of 2D gaussians (reference: src/rtgs/core/gaussians2d.py:1-115).

Cholesky parameterisation L = [[l11, 0], [l21, l22]], Sigma = L L^T, packed as (l11, l21, l22);
RGB ``color`` in [0, 1] times a scalar ``weight`` in [0, 1] (accumulated, not alpha).
"""

from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch


def chol_matrix(chol: torch.Tensor) -> torch.Tensor:
    """(..., 2, 2) lower-triangular factors from packed (..., 3) (gaussians2d.py:21-25)."""
    l11, l21, l22 = chol[..., 0], chol[..., 1], chol[..., 2]
    zero = torch.zeros_like(l11)
    row0 = torch.stack([l11, zero], -1)
    row1 = torch.stack([l21, l22], -1)
    return torch.stack([row0, row1], dim=-2)


def chol_covariance(chol: torch.Tensor) -> torch.Tensor:
    """(..., 2, 2) Sigma = L L^T (gaussians2d.py:28-31)."""
    lmat = chol_matrix(chol)
    return lmat @ lmat.transpose(-1, -2)


def chol_inverse_covariance(chol: torch.Tensor) -> torch.Tensor:
    """(..., 2, 2) analytic Sigma^-1 (gaussians2d.py:34-44)."""
    l11, l21, l22 = chol[..., 0], chol[..., 1], chol[..., 2]
    inv_l11 = 1.0 / l11
    off = -l21 / (l11 * l22)
    inv_l22 = 1.0 / l22
    i00 = inv_l11 * inv_l11 + off * off
    i01 = off * inv_l22
    i11 = inv_l22 * inv_l22
    return torch.stack([torch.stack([i00, i01], -1), torch.stack([i01, i11], -1)], dim=-2)


@dataclass
class Gaussians2D:
    """N 2D gaussians in pixel coordinates of one image (gaussians2d.py:47-115)."""

    xy: torch.Tensor  # (N, 2)
    chol: torch.Tensor  # (N, 3) (l11, l21, l22), l11 > 0, l22 > 0
    color: torch.Tensor  # (N, 3) in [0, 1]
    weight: torch.Tensor  # (N,) in [0, 1]

    def __post_init__(self) -> None:
        n = self.xy.shape[0]
        if self.chol.shape != (n, 3) or self.color.shape != (n, 3) or self.weight.shape != (n,):
            raise ValueError("inconsistent Gaussians2D field shapes")

    @property
    def n(self) -> int:
        return self.xy.shape[0]

    def cholesky_matrix(self) -> torch.Tensor:
        return chol_matrix(self.chol)

    def covariance(self) -> torch.Tensor:
        return chol_covariance(self.chol)

    def inverse_covariance(self) -> torch.Tensor:
        return chol_inverse_covariance(self.chol)

    def detach(self) -> Gaussians2D:
        return Gaussians2D(
            self.xy.detach().clone(),
            self.chol.detach().clone(),
            self.color.detach().clone(),
            self.weight.detach().clone(),
        )

    def to(self, device: torch.device | str) -> Gaussians2D:
        return Gaussians2D(
            self.xy.to(device), self.chol.to(device), self.color.to(device), self.weight.to(device)
        )

    def save_npz(self, path: str | Path) -> None:
        np.savez_compressed(
            Path(path),
            xy=self.xy.detach().cpu().numpy(),
            chol=self.chol.detach().cpu().numpy(),
            color=self.color.detach().cpu().numpy(),
            weight=self.weight.detach().cpu().numpy(),
        )

    @staticmethod
    def load_npz(path: str | Path) -> Gaussians2D:
        data = np.load(Path(path))
        return Gaussians2D(
            xy=torch.from_numpy(data["xy"]).float(),
            chol=torch.from_numpy(data["chol"]).float(),
            color=torch.from_numpy(data["color"]).float(),
            weight=torch.from_numpy(data["weight"]).float(),
        )
