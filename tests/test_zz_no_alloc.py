"""The allocation-free forward entry point (rtgs2d_forward_noalloc) against rtgs2d_forward.

This file is collected last on purpose: if it fails, a run that stops at the first failure has
already run every other test. It passes alone in a fresh process and after the other tests (it
depends on no state they leave behind).

Callers of rtgs2d_forward_noalloc are those that may not allocate device memory (a plugin inside
a host application that owns all device memory, a latency-critical loop where cudaMalloc would
synchronise the device, a process whose free memory another allocator already holds); its
scratch is a 32 MiB static device array shared by all calls. Tolerance: the same 1e-5 relative
error as the other render tests (the two entry points run the same kernels, so the outputs are
expected to be bit-identical).
"""

from __future__ import annotations

import pytest
import torch

from conftest import rel_err
from gpu_helpers import DEV, cuda, stacked
from oracle import render2d as orender
from rtgs_b200 import _native

pytestmark = pytest.mark.gpu
RENDER_TOL = 1e-5


def _inputs(seed, views, n, h, w):
    xy, chol, color, weight = stacked(seed, views, n, h, w, margin=6.0, hi=6.0, off=1.0)
    xy_f, chol_f = xy.reshape(-1, 2), chol.reshape(-1, 3)
    conics = orender.chol_conics(chol_f)
    rects = orender.cuda_rects(xy_f, chol_f, h, w)
    view = torch.arange(views, dtype=torch.int32).repeat_interleave(n)
    return cuda(xy_f, conics, color.reshape(-1, 3), weight.reshape(-1), rects, view)


def _render(fn_name, d, m, views, h, w, with_den):
    lib = _native.lib()
    out = torch.full((views, h, w, 3), float("nan"), device=DEV)
    den = torch.full((views, h, w), float("nan"), device=DEV) if with_den else None
    args = [x.data_ptr() for x in d] + [m, views, h, w, 12.0, out.data_ptr(), _native.ptr(den), None]
    if fn_name == "rtgs2d_forward":
        rc = lib.rtgs2d_forward(_native.arena(DEV), *args)
    else:
        rc = lib.rtgs2d_forward_noalloc(*args)
    _native.check(rc)
    torch.cuda.synchronize()
    return out, den


def test_noalloc_forward_matches_arena_forward_on_consecutive_calls():
    cases = [(31, 2, 400, 45, 61, True), (32, 3, 1500, 96, 130, False), (33, 1, 0, 16, 16, True)]
    for seed, views, n, h, w, with_den in cases:
        d = _inputs(seed, views, n, h, w)
        m = views * n
        ref_out, ref_den = _render("rtgs2d_forward", d, m, views, h, w, with_den)
        for _ in range(2):  # two calls in a row share the static scratch
            out, den = _render("rtgs2d_forward_noalloc", d, m, views, h, w, with_den)
            assert rel_err(out, ref_out) <= RENDER_TOL
            assert torch.isfinite(out).all()
            if with_den:
                assert rel_err(den, ref_den) <= RENDER_TOL


def _crowded_tile_inputs(seed, n_extra, h, w):
    """Random gaussians plus n_extra tiny ones inside tile (1, 1): a tile list longer than the
    per-tile sort, so both entry points bin by the radix sort."""
    xy, chol, color, weight = stacked(seed, 1, 400, h, w, margin=6.0, hi=5.0, off=1.0)
    gen = torch.Generator().manual_seed(seed + 1)
    xy2 = 18.0 + 12.0 * torch.rand(1, n_extra, 2, generator=gen)
    chol2 = torch.zeros(1, n_extra, 3)
    chol2[..., 0] = 0.4 + 0.3 * torch.rand(1, n_extra, generator=gen)
    chol2[..., 2] = 0.4 + 0.3 * torch.rand(1, n_extra, generator=gen)
    xy, chol = torch.cat([xy, xy2], 1), torch.cat([chol, chol2], 1)
    color = torch.cat([color, torch.rand(1, n_extra, 3, generator=gen)], 1)
    weight = torch.cat([weight, torch.rand(1, n_extra, generator=gen)], 1)
    xy_f, chol_f = xy.reshape(-1, 2), chol.reshape(-1, 3)
    view = torch.zeros(xy_f.shape[0], dtype=torch.int32)
    return cuda(xy_f, orender.chol_conics(chol_f), color.reshape(-1, 3), weight.reshape(-1),
                orender.cuda_rects(xy_f, chol_f, h, w), view)


def test_noalloc_radix_and_many_tile_paths_are_bit_identical_to_the_arena_forward():
    """The static scratch is carved differently on the radix path (entry double buffer) and on
    frames with more tiles than the single-block tile scan (device-wide scan temporaries)."""
    crowded = (_crowded_tile_inputs(40, 3000, 64, 80), 1, 64, 80)
    many = (_inputs(41, 2, 3000, 1040, 1100), 2, 1040, 1100)  # 2 x 65 x 69 = 8,970 tiles
    for d, views, h, w in (crowded, many):
        m = d[0].shape[0]
        ref_out, ref_den = _render("rtgs2d_forward", d, m, views, h, w, True)
        for _ in range(2):
            out, den = _render("rtgs2d_forward_noalloc", d, m, views, h, w, True)
            assert torch.equal(out, ref_out) and torch.equal(den, ref_den)


def test_noalloc_forward_allocates_no_device_memory():
    """After the first call on the device (which commits the static array), further calls leave
    the device's free memory unchanged: outputs are the caller's, scratch is the static array."""
    views, n, h, w = 2, 1500, 96, 130
    d = _inputs(42, views, n, h, w)
    out = torch.empty(views, h, w, 3, device=DEV)
    den = torch.empty(views, h, w, device=DEV)
    lib = _native.lib()
    args = [x.data_ptr() for x in d] + [views * n, views, h, w, 12.0, out.data_ptr(), den.data_ptr(), None]
    _native.check(lib.rtgs2d_forward_noalloc(*args))
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info(DEV)
    for _ in range(3):
        _native.check(lib.rtgs2d_forward_noalloc(*args))
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info(DEV)
    assert free_after == free_before


def test_noalloc_forward_rejects_problems_beyond_its_scratch():
    m, h, w = 600_000, 64, 64  # ~45 MB of per-gaussian scratch > 32 MiB
    d = _inputs(34, 1, m, h, w)
    lib = _native.lib()
    out = torch.zeros(1, h, w, 3, device=DEV)
    rc = lib.rtgs2d_forward_noalloc(*(x.data_ptr() for x in d), m, 1, h, w, 12.0, out.data_ptr(), None, None)
    assert rc == -4
    assert b"32 MiB" in lib.rtgs2d_last_error()
    torch.cuda.synchronize()
