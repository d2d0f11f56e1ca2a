"""Load 2D gaussian image archives (``.npz``) into ``Gaussians2D``
(reference: src/rtgs/image2gs/adapters.py:13-82, same entry point and conventions).

Three archive layouts are read:
  native         xy (N,2), chol (N,3), color (N,3), weight (N,): this package's own
                 ``Gaussians2D.save_npz`` files, returned unchanged;
  structsplat    means (N,2) with pixel centres at integer coordinates, log_scales (N,2),
                 rotations (N,) in radians, colors (N,3) (may leave [0,1]), optional
                 opacities (logits) and filter_variance (added to both variances);
  gaussianimage  GaussianImage-style fields under common names: means | xy | positions,
                 colors | color | rgb, log_scales or scales | scale | scaling (one column =
                 isotropic), rotations | rotation | angles | angle, and opacities (logits) |
                 opacity | weight (clamped to [0,1]); weight 1 when absent.
``source="auto"`` picks native when the four native fields are present, else structsplat when
means, log_scales, rotations and colors are, else gaussianimage. Geometry converts exactly up to
float rounding: pixel centres move from integer to half-integer coordinates (structsplat only)
and the rotation-scale covariance R diag(s^2) R^T (+ 1e-8 on the diagonal, as the reference)
becomes its Cholesky factor; colours are clamped to [0,1].
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

from rtgs_b200.core.gaussians2d import Gaussians2D

NATIVE_FIELDS = ("xy", "chol", "color", "weight")
STRUCTSPLAT_FIELDS = ("means", "log_scales", "rotations", "colors")
# Accepted names per quantity, in order of preference.
FIELD_NAMES = {
    "mean": ("means", "xy", "positions"),
    "color": ("colors", "color", "rgb"),
    "scale": ("scales", "scale", "scaling"),
    "angle": ("rotations", "rotation", "angles", "angle"),
}
COVARIANCE_JITTER = 1e-8


def detect_source(fields) -> str:
    """The layout ``source="auto"`` resolves to for an archive with these field names."""
    names = set(fields)
    if set(NATIVE_FIELDS) <= names:
        return "native"
    if set(STRUCTSPLAT_FIELDS) <= names:
        return "structsplat"
    return "gaussianimage"


def load_gaussians2d(path: str | Path, source: str = "auto") -> Gaussians2D:
    """Read a native, StructSplat or GaussianImage-style ``.npz`` archive (float32, CPU)."""
    with np.load(Path(path)) as archive:
        arrays = {name: np.asarray(archive[name]) for name in archive.files}
    return gaussians_from_arrays(arrays, source)


def gaussians_from_arrays(arrays: dict[str, np.ndarray], source: str = "auto") -> Gaussians2D:
    """``load_gaussians2d`` on an already loaded name -> array mapping."""
    if source == "auto":
        source = detect_source(arrays)
    if source == "native":
        return Gaussians2D(*(_f32(arrays[name]) for name in NATIVE_FIELDS))
    means = _pick(arrays, "mean").astype(np.float32)
    if source == "structsplat":
        means = means + np.float32(0.5)
    colors = np.clip(_pick(arrays, "color").astype(np.float32), 0.0, 1.0)
    if "log_scales" in arrays:
        scales = np.exp(arrays["log_scales"].astype(np.float32))
    else:
        scales = _pick(arrays, "scale").astype(np.float32)
    if source == "structsplat" and "filter_variance" in arrays:
        extra = np.maximum(arrays["filter_variance"].astype(np.float32).reshape(-1, 1), 0.0)
        scales = np.sqrt(scales * scales + extra)
    angles = _pick(arrays, "angle").astype(np.float32).reshape(-1)
    chol = rotation_scale_cholesky(scales, angles)
    weight = _weights(arrays, means.shape[0])
    return Gaussians2D(_f32(means), torch.from_numpy(chol), _f32(colors), _f32(weight))


def rotation_scale_cholesky(scales: np.ndarray, angles: np.ndarray) -> np.ndarray:
    """(N,3) float32 (l11, l21, l22): the Cholesky factor of R(angle) diag(s^2) R(angle)^T plus
    COVARIANCE_JITTER on the diagonal, in closed form (evaluated in float64). ``scales`` is
    (N,2) or (N,) / (N,1) for isotropic gaussians."""
    s = np.asarray(scales, dtype=np.float64)
    if s.ndim == 1 or s.shape[-1] == 1:
        s = np.repeat(s.reshape(-1, 1), 2, axis=1)
    a, b = s[:, 0] ** 2, s[:, 1] ** 2
    c, sn = np.cos(np.asarray(angles, dtype=np.float64)), np.sin(np.asarray(angles, dtype=np.float64))
    s00 = c * c * a + sn * sn * b + COVARIANCE_JITTER
    s01 = c * sn * (a - b)
    s11 = sn * sn * a + c * c * b + COVARIANCE_JITTER
    l11 = np.sqrt(s00)
    l21 = s01 / l11
    l22 = np.sqrt(s11 - l21 * l21)
    return np.stack([l11, l21, l22], axis=-1).astype(np.float32)


def _weights(arrays: dict[str, np.ndarray], n: int) -> np.ndarray:
    if "opacities" in arrays:  # logits
        return (1.0 / (1.0 + np.exp(-arrays["opacities"].astype(np.float64)))).astype(np.float32).reshape(-1)
    for name in ("opacity", "weight"):
        if name in arrays:
            return np.clip(arrays[name].astype(np.float32).reshape(-1), 0.0, 1.0)
    return np.ones(n, dtype=np.float32)


def _pick(arrays: dict[str, np.ndarray], quantity: str) -> np.ndarray:
    for name in FIELD_NAMES[quantity]:
        if name in arrays:
            return arrays[name]
    raise ValueError(f"2D Gaussian archive is missing one of: {', '.join(FIELD_NAMES[quantity])}")


def _f32(array: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.array(array, dtype=np.float32, copy=True))
