"""ctypes binding of librtgs2d.so (the C ABI declared in include/rtgs2d.h).

Loading is lazy: importing this package never touches CUDA. Every entry point raises
RuntimeError with the library's message when a call fails, and RuntimeError when the library
has not been built -- there is no CPU fallback.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "librtgs2d.so"

_c_int64 = ctypes.c_int64
_vp = ctypes.c_void_p
_dbl = ctypes.c_double

LOSS_MSE = 0
LOSS_MASK_WEIGHTED = 1
LOSS_MASK_ONLY = 2

INIT_NONFINITE_RAW = 256  # RTGS2D_INIT_NONFINITE_RAW of rtgs2d_fit_set_initial

APPEARANCE_WEIGHT_COLOR_9P = 0  # RTGS2D_APPEARANCE_* of rtgs2d_fit_set_appearance
APPEARANCE_UNIT_WEIGHT_8P = 1


class FitOptions(ctypes.Structure):
    _fields_ = [
        ("lr", ctypes.c_double),
        ("iterations", ctypes.c_int64),
        ("log_every", ctypes.c_int64),
        ("check_every", ctypes.c_int64),
        ("freeze_geometry", ctypes.c_int32),
        ("loss_mode", ctypes.c_int32),
        ("mask_coverage_weight", ctypes.c_double),
    ]


_SIGNATURES = {
    "rtgs2d_abi_version": ([], ctypes.c_int),
    "rtgs2d_last_error": ([], ctypes.c_char_p),
    "rtgs2d_arena_create": ([ctypes.POINTER(_vp)], ctypes.c_int),
    "rtgs2d_arena_destroy": ([_vp], ctypes.c_int),
    "rtgs2d_arena_last_stats": ([_vp, ctypes.POINTER(_c_int64), ctypes.POINTER(_c_int64)], ctypes.c_int),
    "rtgs2d_forward": (
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _c_int64, _c_int64, _c_int64, _c_int64, _dbl, _vp, _vp, _vp],
        ctypes.c_int,
    ),
    "rtgs2d_backward": (
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _c_int64, _c_int64, _c_int64, _c_int64, _dbl,
         _vp, _vp, _vp, _vp, _vp],
        ctypes.c_int,
    ),
    "rtgs2d_forward_noalloc": (
        [_vp, _vp, _vp, _vp, _vp, _vp, _c_int64, _c_int64, _c_int64, _c_int64, _dbl, _vp, _vp, _vp],
        ctypes.c_int,
    ),
    "rtgs2d_render_forward": (
        [_vp, _vp, _vp, _vp, _vp, _c_int64, _c_int64, _c_int64, _c_int64, _vp, _vp, _vp],
        ctypes.c_int,
    ),
    "rtgs2d_render_backward": (
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _c_int64, _c_int64, _c_int64, _c_int64, _vp, _vp, _vp, _vp, _vp],
        ctypes.c_int,
    ),
    "rtgs2d_render_backward_after_forward": (
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _c_int64, _c_int64, _c_int64, _c_int64, _vp, _vp, _vp, _vp, _vp],
        ctypes.c_int,
    ),
    "rtgs2d_support_rects": ([_vp, _vp, _c_int64, _c_int64, _c_int64, _vp, _vp, _vp], ctypes.c_int),
    "rtgs2d_arena_copy_binning": (
        [_vp, _c_int64, _vp, _c_int64, _vp, ctypes.POINTER(_c_int64), ctypes.POINTER(_c_int64), _vp],
        ctypes.c_int,
    ),
    "rtgs2d_fit_create": (
        [_c_int64, _c_int64, _c_int64, _c_int64, ctypes.POINTER(FitOptions), ctypes.POINTER(_vp)],
        ctypes.c_int,
    ),
    "rtgs2d_fit_destroy": ([_vp], ctypes.c_int),
    "rtgs2d_fit_set_targets": ([_vp, _vp, _vp, _vp], ctypes.c_int),
    "rtgs2d_fit_set_raw": ([_vp, _vp, _vp, _vp, _vp, _vp, _vp], ctypes.c_int),
    "rtgs2d_fit_set_initial": ([_vp, _vp, _vp, _vp, _vp, _vp, _vp], ctypes.c_int),
    "rtgs2d_fit_set_appearance": ([_vp, ctypes.c_int32], ctypes.c_int),
    "rtgs2d_fit_run": ([_vp, _c_int64, _vp], ctypes.c_int),
    "rtgs2d_fit_get_raw": ([_vp, _vp, _vp, _vp, _vp, _vp, _vp], ctypes.c_int),
    "rtgs2d_fit_get_params": ([_vp, _vp, _vp, _vp, _vp, _vp], ctypes.c_int),
    "rtgs2d_fit_evaluate": ([_vp, _vp, _vp, _vp], ctypes.c_int),
    "rtgs2d_fit_gradients": ([_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp], ctypes.c_int),
    "rtgs2d_fit_get_moments": ([_vp, ctypes.c_int32, _vp, _vp, _vp, _vp, _vp, _vp], ctypes.c_int),
    "rtgs2d_fit_history": ([_vp, _c_int64, _vp, _vp, ctypes.POINTER(_c_int64)], ctypes.c_int),
    "rtgs2d_fit_set_profiling": ([_vp, ctypes.c_int32], ctypes.c_int),
    "rtgs2d_fit_set_graphs": ([_vp, ctypes.c_int32], ctypes.c_int),
    "rtgs2d_fit_set_binning": ([_vp, ctypes.c_int32], ctypes.c_int),
    "rtgs2d_fit_set_active": ([_vp, _vp, _vp], ctypes.c_int),
    "rtgs2d_fit_write_rows": ([_vp, _vp, _c_int64, _vp, _vp, _vp, _vp, _vp, _vp], ctypes.c_int),
    "rtgs2d_fit_chunk_counts": ([_vp, ctypes.POINTER(_c_int64), ctypes.POINTER(_c_int64)], ctypes.c_int),
    "rtgs2d_fit_reserve": ([_vp, _c_int64, _vp], ctypes.c_int),
    "rtgs2d_fit_capacity": ([_vp, ctypes.POINTER(_c_int64), ctypes.POINTER(_c_int64)], ctypes.c_int),
    "rtgs2d_fit_stage_times": (
        [_vp, ctypes.POINTER(_dbl), ctypes.POINTER(_dbl), ctypes.POINTER(_dbl), ctypes.POINTER(_c_int64),
         ctypes.POINTER(_dbl)],
        ctypes.c_int,
    ),
    "rtgs2d_adam_step": (
        [ctypes.c_int32, _vp, _vp, _vp, _vp, _vp, _dbl, _dbl, _dbl, _dbl, _c_int64, _vp],
        ctypes.c_int,
    ),
    "rtgs2d_fit_stats": (
        [_vp, ctypes.POINTER(_c_int64), ctypes.POINTER(_c_int64), ctypes.POINTER(_c_int64),
         ctypes.POINTER(ctypes.c_double)],
        ctypes.c_int,
    ),
}

_LIB: ctypes.CDLL | None = None
_LOCK = threading.Lock()
_ARENAS: dict[int, int] = {}


def exported_symbols() -> tuple[str, ...]:
    """Names of the C entry points this binding declares (all of include/rtgs2d.h)."""
    return tuple(_SIGNATURES)


def lib() -> ctypes.CDLL:
    """Load librtgs2d.so once; raise if it is missing (no fallback path exists)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    with _LOCK:
        if _LIB is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"the rtgs_b200 CUDA library is not built ({LIB_PATH} missing); run "
                    "`python -m rtgs_b200._build` or __graft_entry__.build()"
                )
            handle = ctypes.CDLL(str(LIB_PATH))
            for name, (argtypes, restype) in _SIGNATURES.items():
                fn = getattr(handle, name)
                fn.argtypes = argtypes
                fn.restype = restype
            _LIB = handle
    return _LIB


def check(rc: int) -> None:
    if rc != 0:
        msg = lib().rtgs2d_last_error()
        raise RuntimeError(f"rtgs2d error {rc}: {msg.decode() if msg else 'unknown'}")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def arena(device: torch.device) -> int:
    """Per-device scratch arena (created on first use, lives for the process)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    with _LOCK:
        handle = _ARENAS.get(idx)
    if handle is not None:
        return handle
    out = _vp()
    with torch.cuda.device(idx):
        check(lib().rtgs2d_arena_create(ctypes.byref(out)))
    with _LOCK:
        _ARENAS.setdefault(idx, out.value)
        return _ARENAS[idx]


def arena_last_stats(device: torch.device) -> tuple[int, int]:
    e, p = _c_int64(), _c_int64()
    check(lib().rtgs2d_arena_last_stats(arena(device), ctypes.byref(e), ctypes.byref(p)))
    return int(e.value), int(p.value)
