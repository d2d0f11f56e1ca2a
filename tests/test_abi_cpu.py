"""The C-ABI library loads and exports every entry point that include/rtgs2d.h declares.

No compute call is made: these tests run on machines without a GPU.
"""

from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

from conftest import ROOT
from rtgs_b200 import _native

HEADER = ROOT / "include" / "rtgs2d.h"


def _declared() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"^RTGS2D_API\s+[\w\s\*]+?\b(rtgs2d_\w+)\s*\(", text, flags=re.M))


def test_header_declares_the_binding_surface():
    declared = _declared()
    assert len(declared) >= 20
    assert declared == set(_native.exported_symbols())


def test_library_exports_every_declared_symbol():
    lib = _native.lib()
    for name in _declared():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(_native.LIB_PATH)], capture_output=True, text=True)
    exported = set(re.findall(r"\b(rtgs2d_\w+)\b", out.stdout))
    assert _declared() <= exported


def test_build_targets_sm_100a_only():
    from rtgs_b200 import _build

    assert _build.ARCH_FLAGS == ["-gencode", "arch=compute_100a,code=sm_100a"]


def test_version_and_error_string_need_no_gpu():
    lib = _native.lib()
    assert lib.rtgs2d_abi_version() == 2
    assert isinstance(lib.rtgs2d_last_error(), bytes)


def test_null_arguments_are_rejected_before_any_device_work():
    lib = _native.lib()
    rc = lib.rtgs2d_arena_create(None)
    assert rc == -1
    assert b"NULL" in lib.rtgs2d_last_error()
    rc = lib.rtgs2d_fit_create(1, 4, 8, 8, None, ctypes.byref(ctypes.c_void_p()))
    assert rc == -1
