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


def test_noalloc_forward_rejects_problems_beyond_its_scratch():
    m, h, w = 600_000, 64, 64  # ~45 MB of per-gaussian scratch > 32 MiB
    d = _inputs(34, 1, m, h, w)
    lib = _native.lib()
    out = torch.zeros(1, h, w, 3, device=DEV)
    rc = lib.rtgs2d_forward_noalloc(*(x.data_ptr() for x in d), m, 1, h, w, 12.0, out.data_ptr(), None, None)
    assert rc == -4
    assert b"32 MiB" in lib.rtgs2d_last_error()
    torch.cuda.synchronize()
