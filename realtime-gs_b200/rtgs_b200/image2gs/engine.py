"""Python handle over the C fit engine (rtgs2d_fit_* in include/rtgs2d.h).

The whole iteration loop runs in C++/CUDA; Python only moves tensors in and out.
"""

from __future__ import annotations

import collections
import ctypes
import math
import threading

import numpy as np
import torch

from rtgs_b200 import _native

_RAW_SHAPES = (("xy_raw", 2), ("diag_raw", 2), ("off_raw", 0), ("color_raw", 3), ("weight_raw", 0))
# unit_weight_bounded_8p: the colour slots hold amplitude_raw and there is no weight parameter
_RAW_SHAPES_8P = (("xy_raw", 2), ("diag_raw", 2), ("off_raw", 0), ("amplitude_raw", 3))
WEIGHT_COLOR_9P = "weight_color_9p"
UNIT_WEIGHT_8P = "unit_weight_bounded_8p"
_APPEARANCE_CODES = {WEIGHT_COLOR_9P: _native.APPEARANCE_WEIGHT_COLOR_9P,
                     UNIT_WEIGHT_8P: _native.APPEARANCE_UNIT_WEIGHT_8P}


def pack_mask_bits(masks: torch.Tensor) -> torch.Tensor:
    """(B, H, W) masks -> (B, ceil(H*W/8)) uint8, bit i of byte k = pixel 8k+i (little-endian).

    Same bit order as numpy ``packbits(bitorder="little")`` used by the reference's PackedAlpha
    (src/rtgs/data/compact_views.py:279-284). A pixel is in the mask when its value is > 0.5.
    """
    b = masks.shape[0]
    flat = (masks.reshape(b, -1) > 0.5).to(torch.uint8)
    pad = (-flat.shape[1]) % 8
    if pad:
        flat = torch.cat([flat, flat.new_zeros(b, pad)], dim=1)
    weights = (2 ** torch.arange(8, device=flat.device, dtype=torch.int32)).to(torch.uint8)
    return (flat.reshape(b, -1, 8) * weights).sum(dim=2, dtype=torch.int32).to(torch.uint8).contiguous()


class FitEngine:
    """Device-resident fit state for B views x N gaussians of an H x W image."""

    def __init__(
        self,
        n_views: int,
        n: int,
        height: int,
        width: int,
        *,
        lr: float,
        iterations: int,
        log_every: int,
        check_every: int = 0,
        freeze_geometry: bool = False,
        loss_mode: int = _native.LOSS_MSE,
        device: torch.device | None = None,
        mask_coverage_weight: float = 0.0,
        appearance: str = WEIGHT_COLOR_9P,
    ) -> None:
        if appearance not in _APPEARANCE_CODES:
            raise ValueError(f"unknown appearance parameterization {appearance!r}")
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.n_views, self.n, self.height, self.width = int(n_views), int(n), int(height), int(width)
        self.iterations = int(iterations)
        opts = _native.FitOptions(
            lr=float(lr), iterations=int(iterations), log_every=int(log_every),
            check_every=int(check_every), freeze_geometry=int(bool(freeze_geometry)),
            loss_mode=int(loss_mode), mask_coverage_weight=float(mask_coverage_weight),
        )
        self._lib = _native.lib()
        handle = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _native.check(
                self._lib.rtgs2d_fit_create(self.n_views, self.n, self.height, self.width,
                                            ctypes.byref(opts), ctypes.byref(handle))
            )
        self._h = handle.value
        self.appearance = appearance
        self._raw_shapes = _RAW_SHAPES_8P if appearance == UNIT_WEIGHT_8P else _RAW_SHAPES
        _native.check(self._lib.rtgs2d_fit_set_appearance(self._h, _APPEARANCE_CODES[appearance]))

    # -- lifecycle -------------------------------------------------------------------------------
    def close(self) -> None:
        if getattr(self, "_h", None):
            with torch.cuda.device(self.device):
                self._lib.rtgs2d_fit_destroy(self._h)
            self._h = None

    def __del__(self) -> None:  # pragma: no cover - interpreter shutdown order
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self) -> FitEngine:
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def _stream(self) -> int:
        return _native.stream_ptr(self.device)

    # -- inputs ----------------------------------------------------------------------------------
    def set_targets(self, targets: torch.Tensor, mask_bits: torch.Tensor | None = None) -> None:
        targets = targets.to(self.device, torch.float32).contiguous()
        if targets.shape != (self.n_views, self.height, self.width, 3):
            raise ValueError("targets must be (B, H, W, 3)")
        if mask_bits is not None:
            mask_bits = mask_bits.to(self.device, torch.uint8).contiguous()
        with torch.cuda.device(self.device):
            _native.check(
                self._lib.rtgs2d_fit_set_targets(self._h, targets.data_ptr(), _native.ptr(mask_bits), self._stream())
            )

    def set_raw(self, raw: dict[str, torch.Tensor]) -> None:
        """Raw parameters by name: xy_raw, diag_raw, off_raw and color_raw + weight_raw, or
        amplitude_raw for the unit-weight appearance."""
        ts = []
        for name, k in self._raw_shapes:
            t = raw[name].to(self.device, torch.float32).contiguous()
            want = (self.n_views, self.n, k) if k else (self.n_views, self.n)
            if tuple(t.shape) != want:
                raise ValueError(f"{name} must have shape {want}, got {tuple(t.shape)}")
            ts.append(t)
        ptrs = [t.data_ptr() for t in ts] + [None] * (5 - len(ts))
        with torch.cuda.device(self.device):
            _native.check(self._lib.rtgs2d_fit_set_raw(self._h, *ptrs, self._stream()))
            torch.cuda.current_stream(self.device).synchronize()

    def set_initial(self, xy: torch.Tensor, chol: torch.Tensor, color: torch.Tensor,
                    weight: torch.Tensor) -> int:
        """Validate and transform constrained (B, N, .) initial parameters on the device
        (rtgs2d_fit_set_initial); returns 0 or the RTGS2D_INIT_* bits of the failed checks."""
        b, n = self.n_views, self.n
        ts = []
        for t, k in ((xy, 2), (chol, 3), (color, 3), (weight, 0)):
            t = t.to(self.device, torch.float32).contiguous()
            want = (b, n, k) if k else (b, n)
            if t.numel() != b * n * max(k, 1):
                raise ValueError(f"initial parameters must have {want} elements, got {tuple(t.shape)}")
            ts.append(t)
        status = ctypes.c_uint32()
        with torch.cuda.device(self.device):
            _native.check(self._lib.rtgs2d_fit_set_initial(self._h, *(t.data_ptr() for t in ts),
                                                           ctypes.byref(status), self._stream()))
        return int(status.value)

    # -- running ---------------------------------------------------------------------------------
    def run(self, n_iterations: int) -> None:
        with torch.cuda.device(self.device):
            _native.check(self._lib.rtgs2d_fit_run(self._h, int(n_iterations), self._stream()))

    def params(self) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
        b, n = self.n_views, self.n
        kw = dict(device=self.device, dtype=torch.float32)
        xy = torch.empty(b, n, 2, **kw)
        chol = torch.empty(b, n, 3, **kw)
        color = torch.empty(b, n, 3, **kw)
        weight = torch.empty(b, n, **kw)
        with torch.cuda.device(self.device):
            _native.check(
                self._lib.rtgs2d_fit_get_params(self._h, xy.data_ptr(), chol.data_ptr(), color.data_ptr(),
                                                weight.data_ptr(), self._stream())
            )
        return xy, chol, color, weight

    def raw(self) -> dict[str, torch.Tensor]:
        out = self._raw_like()
        ptrs = [t.data_ptr() for t in out.values()] + [None] * (5 - len(out))
        with torch.cuda.device(self.device):
            _native.check(self._lib.rtgs2d_fit_get_raw(self._h, *ptrs, self._stream()))
        return out

    def _raw_like(self) -> dict[str, torch.Tensor]:
        b, n = self.n_views, self.n
        return {name: torch.empty((b, n, k) if k else (b, n), device=self.device, dtype=torch.float32)
                for name, k in self._raw_shapes}

    def gradients(self, want_render: bool = True) -> tuple[dict[str, torch.Tensor], torch.Tensor | None, np.ndarray]:
        """The fit loss's raw-parameter gradients at the current state, without an update
        (rtgs2d_fit_gradients); returns (gradients by raw name, render (B,H,W,3) or None, sums (B,2))."""
        grads = self._raw_like()
        render = None
        if want_render:
            render = torch.empty(self.n_views, self.height, self.width, 3, device=self.device, dtype=torch.float32)
        sums = np.zeros((self.n_views, 2), dtype=np.float64)
        ptrs = [t.data_ptr() for t in grads.values()] + [None] * (5 - len(grads))
        with torch.cuda.device(self.device):
            _native.check(self._lib.rtgs2d_fit_gradients(self._h, *ptrs, _native.ptr(render), sums.ctypes.data,
                                                         self._stream()))
        return grads, render, sums

    def moments(self) -> tuple[dict[str, torch.Tensor], dict[str, torch.Tensor]]:
        """Adam's (exp_avg, exp_avg_sq) by raw parameter name (rtgs2d_fit_get_moments)."""
        out = []
        for which in (1, 2):
            m = self._raw_like()
            ptrs = [t.data_ptr() for t in m.values()] + [None] * (5 - len(m))
            with torch.cuda.device(self.device):
                _native.check(self._lib.rtgs2d_fit_get_moments(self._h, which, *ptrs, self._stream()))
            out.append(m)
        return out[0], out[1]

    def evaluate(self, want_render: bool = True) -> tuple[torch.Tensor | None, np.ndarray]:
        """Render the current parameters; returns (render (B,H,W,3) or None, sums (B, 2))."""
        render = None
        if want_render:
            render = torch.empty(self.n_views, self.height, self.width, 3, device=self.device, dtype=torch.float32)
        sums = np.zeros((self.n_views, 2), dtype=np.float64)
        with torch.cuda.device(self.device):
            _native.check(
                self._lib.rtgs2d_fit_evaluate(self._h, _native.ptr(render), sums.ctypes.data, self._stream())
            )
        return render, sums

    def history(self) -> tuple[np.ndarray, np.ndarray]:
        """(iterations (R,), sums (R, B, 2)) recorded so far."""
        n_rows = ctypes.c_int64()
        _native.check(self._lib.rtgs2d_fit_history(self._h, 0, None, None, ctypes.byref(n_rows)))
        rows = int(n_rows.value)
        iters = np.zeros(rows, dtype=np.int64)
        sums = np.zeros((rows, self.n_views, 2), dtype=np.float64)
        if rows:
            with torch.cuda.device(self.device):
                _native.check(
                    self._lib.rtgs2d_fit_history(self._h, rows, iters.ctypes.data, sums.ctypes.data, ctypes.byref(n_rows))
                )
        return iters, sums

    def reserve(self, entries: int) -> None:
        """Pre-size the (gaussian, tile) entry capacity of the fit loop."""
        with torch.cuda.device(self.device):
            _native.check(self._lib.rtgs2d_fit_reserve(self._h, int(entries), self._stream()))

    def capacity(self) -> tuple[int, int]:
        """(entry capacity, chunks re-run after a capacity overflow)."""
        e, r = ctypes.c_int64(), ctypes.c_int64()
        _native.check(self._lib.rtgs2d_fit_capacity(self._h, ctypes.byref(e), ctypes.byref(r)))
        return int(e.value), int(r.value)

    def set_profiling(self, enable: bool = True) -> None:
        """Record CUDA events around binning, the raster kernel and Adam in every iteration."""
        _native.check(self._lib.rtgs2d_fit_set_profiling(self._h, int(bool(enable))))

    def set_active(self, active: torch.Tensor | None) -> None:
        """(n_views, n) bool/uint8 CUDA mask of live rows (parked rows are not rendered); None = all."""
        with torch.cuda.device(self.device):
            if active is None:
                _native.check(self._lib.rtgs2d_fit_set_active(self._h, None, self._stream()))
                return
            if active.shape != (self.n_views, self.n) or active.device != self.device:
                raise ValueError("active mask must be a (n_views, n) tensor on the engine's device")
            a = active.to(torch.uint8).contiguous()
            # `a` is freed on return; the caching allocator reuses it only after the copy queued on
            # the same stream.
            _native.check(self._lib.rtgs2d_fit_set_active(self._h, a.data_ptr(), self._stream()))

    def write_rows(self, rows: torch.Tensor, raw: dict[str, torch.Tensor] | None = None) -> None:
        """Write raw parameters into flat rows (indices into n_views * n) and zero their Adam
        moments; raw = None zeroes the moments only."""
        rows = rows.to(self.device, torch.int64).contiguous()
        n_rows = rows.numel()
        if n_rows == 0:
            return
        ptrs = [None] * 5
        keep = []
        if raw is not None:
            for k, (name, width) in enumerate(self._raw_shapes):
                t = raw[name].to(self.device, torch.float32).reshape(n_rows, max(width, 1)).contiguous()
                keep.append(t)
                ptrs[k] = t.data_ptr()
        with torch.cuda.device(self.device):
            _native.check(self._lib.rtgs2d_fit_write_rows(self._h, rows.data_ptr(), n_rows, *ptrs, self._stream()))

    def set_graphs(self, enable: bool = True) -> None:
        """Replay repeated 64-iteration chunks from a captured CUDA graph (default on)."""
        _native.check(self._lib.rtgs2d_fit_set_graphs(self._h, int(bool(enable))))

    BINNING_MODES = {"auto": 0, "scatter": 1, "radix": 2, "tight": 3, "sorted": 4}

    def set_binning(self, mode: str = "auto") -> None:
        """How the fit loop bins (gaussian, tile) entries; every mode gives identical results.

        "auto": the first iteration of each 64-iteration chunk scatters its entries into tile
        lists, later projections place their ids directly into per-tile segments sized from the
        previous binning (a full segment re-runs the chunk with "scatter") and the fit raster
        sorts each tile's segment itself; "sorted" is "auto" with a separate per-tile sort kernel
        before the raster; "scatter" and "radix" bin every iteration by scatter or by radix sort;
        "tight" is "auto" with segments of exactly the previous counts, which overflow whenever a
        tile gains an entry.
        """
        if mode not in self.BINNING_MODES:
            raise ValueError(f"binning mode must be one of {sorted(self.BINNING_MODES)}, got {mode!r}")
        _native.check(self._lib.rtgs2d_fit_set_binning(self._h, self.BINNING_MODES[mode]))

    def chunk_counts(self) -> tuple[int, int]:
        """(chunks replayed from a CUDA graph, chunks run eagerly) since the engine was created."""
        g, e = ctypes.c_int64(), ctypes.c_int64()
        _native.check(self._lib.rtgs2d_fit_chunk_counts(self._h, ctypes.byref(g), ctypes.byref(e)))
        return int(g.value), int(e.value)

    def stage_times(self) -> dict[str, float]:
        b, r, a, p = ctypes.c_double(), ctypes.c_double(), ctypes.c_double(), ctypes.c_double()
        n = ctypes.c_int64()
        _native.check(self._lib.rtgs2d_fit_stage_times(self._h, ctypes.byref(b), ctypes.byref(r), ctypes.byref(a),
                                                       ctypes.byref(n), ctypes.byref(p)))
        return {"bin_ms": b.value, "raster_ms": r.value, "adam_ms": a.value, "iterations": int(n.value),
                "pairs": p.value}

    def stats(self) -> dict[str, float]:
        step, e, p = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
        total = ctypes.c_double()
        _native.check(self._lib.rtgs2d_fit_stats(self._h, ctypes.byref(step), ctypes.byref(e), ctypes.byref(p), ctypes.byref(total)))
        return {"step": int(step.value), "last_entries": int(e.value), "last_pairs": int(p.value),
                "total_pairs": float(total.value)}


def psnr_values(sums: np.ndarray, counts: np.ndarray) -> list[float]:
    """PSNR (dB) per view from clamped squared-error sums and value counts (metrics.py:12-15)."""
    out = []
    for s, c in zip(sums, counts):
        mse = max(float(s) / float(c), 1e-12) if c > 0 else 1e-12
        out.append(-10.0 * math.log10(mse))
    return out


# ---------------------------------------------------------------------------------------------
# Engine pool. Creating an engine allocates its device buffers and its first run captures the
# CUDA graphs of its chunks; destroying it frees them (cudaFree synchronises the device). Fits that
# repeat one configuration -- the common case when many images are fitted with one FitConfig --
# take an idle engine of that configuration instead, keeping buffers and graphs. A pooled engine
# is reset by set_targets / set_raw, so results do not depend on its history.

_POOL_LOCK = threading.Lock()
_POOL: "collections.OrderedDict[tuple, list[FitEngine]]" = collections.OrderedDict()
_POOL_MAX_IDLE = 4  # idle engines kept per process, least recently released closed first


def acquire_engine(n_views: int, n: int, height: int, width: int, *, lr: float, iterations: int,
                   log_every: int, check_every: int = 0, freeze_geometry: bool = False,
                   loss_mode: int = _native.LOSS_MSE, device: torch.device | None = None,
                   mask_coverage_weight: float = 0.0, appearance: str = WEIGHT_COLOR_9P) -> FitEngine:
    """An idle pooled engine of exactly this configuration, else a new one."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    if dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    key = (dev.index, int(n_views), int(n), int(height), int(width), float(lr), int(iterations),
           int(log_every), int(check_every), bool(freeze_geometry), int(loss_mode),
           float(mask_coverage_weight), str(appearance))
    with _POOL_LOCK:
        idle = _POOL.get(key)
        if idle:
            engine = idle.pop()
            if not idle:
                del _POOL[key]
            return engine
    engine = FitEngine(n_views, n, height, width, lr=lr, iterations=iterations, log_every=log_every,
                       check_every=check_every, freeze_geometry=freeze_geometry, loss_mode=loss_mode,
                       device=dev, mask_coverage_weight=mask_coverage_weight, appearance=appearance)
    engine._pool_key = key
    return engine


def release_engine(engine: FitEngine, reusable: bool = True) -> None:
    """Return an engine from acquire_engine; `reusable=False` (after an error) destroys it."""
    key = getattr(engine, "_pool_key", None)
    if not reusable or key is None or not getattr(engine, "_h", None):
        engine.close()
        return
    evicted = []
    with _POOL_LOCK:
        _POOL.setdefault(key, []).append(engine)
        _POOL.move_to_end(key)
        while sum(len(v) for v in _POOL.values()) > _POOL_MAX_IDLE:
            old_key, old = next(iter(_POOL.items()))
            evicted.append(old.pop(0))
            if not old:
                del _POOL[old_key]
    for e in evicted:
        e.close()


def clear_engine_pool() -> None:
    """Destroy every idle pooled engine (frees their device memory)."""
    with _POOL_LOCK:
        engines = [e for v in _POOL.values() for e in v]
        _POOL.clear()
    for e in engines:
        e.close()

