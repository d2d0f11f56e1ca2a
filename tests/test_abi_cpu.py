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


def _header_defines() -> dict[str, int]:
    text = HEADER.read_text()
    return {m.group(1): int(m.group(2))
            for m in re.finditer(r"^#define RTGS2D_(\w+)\s+\(?(-?\d+)u?\)?", text, flags=re.M)}


def test_python_constants_match_the_header():
    """The binding's copies of the header's loss, appearance, status and binning codes."""
    from rtgs_b200.image2gs.engine import FitEngine

    d = _header_defines()
    for name in ("LOSS_MSE", "LOSS_MASK_WEIGHTED", "LOSS_MASK_ONLY", "APPEARANCE_WEIGHT_COLOR_9P",
                 "APPEARANCE_UNIT_WEIGHT_8P", "INIT_NONFINITE_RAW"):
        assert getattr(_native, name) == d[name], name
    binning = {k[len("BINNING_"):].lower(): v for k, v in d.items() if k.startswith("BINNING_")}
    assert FitEngine.BINNING_MODES == binning
    from rtgs_b200.image2gs import optim

    assert optim.MAX_TENSORS == d["ADAM_MAX_TENSORS"]


def test_fit_options_layout_matches_the_header(tmp_path):
    """ctypes' FitOptions has the C struct's size and field offsets (compiled against the header)."""
    fields = [name for name, _ in _native.FitOptions._fields_]
    src = tmp_path / "layout.c"
    src.write_text(
        "#include <stdio.h>\n#include <stddef.h>\n#include \"rtgs2d.h\"\nint main(void) {\n"
        "  printf(\"size %zu\\n\", sizeof(rtgs2d_fit_options));\n"
        + "".join(f"  printf(\"{f} %zu\\n\", offsetof(rtgs2d_fit_options, {f}));\n" for f in fields)
        + "  return 0;\n}\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c99", "-I", str(HEADER.parent), str(src), "-o", str(exe)], check=True)
    out = dict(line.split() for line in subprocess.run([str(exe)], check=True, capture_output=True,
                                                        text=True).stdout.splitlines())
    assert int(out["size"]) == ctypes.sizeof(_native.FitOptions)
    for f in fields:
        assert int(out[f]) == getattr(_native.FitOptions, f).offset, f


_SCALARS = {"int64_t": ctypes.c_int64, "int32_t": ctypes.c_int32, "int": ctypes.c_int,
            "double": ctypes.c_double, "float": ctypes.c_float, "uint32_t": ctypes.c_uint32,
            "uint64_t": ctypes.c_uint64, "size_t": ctypes.c_size_t}


def _prototypes() -> dict[str, tuple[str, list[str]]]:
    text = re.sub(r"/\*.*?\*/", " ", HEADER.read_text(), flags=re.S)
    protos = {}
    for m in re.finditer(r"^RTGS2D_API\s+([\w\s\*]+?)\s*\b(rtgs2d_\w+)\s*\(([^;]*?)\)\s*;", text, flags=re.M | re.S):
        params = " ".join(m.group(3).split())
        args = [] if params in ("", "void") else [p.strip() for p in params.split(",")]
        protos[m.group(2)] = (" ".join(m.group(1).split()), args)
    return protos


def _is_pointer_type(t) -> bool:
    return t in (ctypes.c_void_p, ctypes.c_char_p) or (isinstance(t, type) and issubclass(t, ctypes._Pointer))


def test_binding_signatures_match_the_header_prototypes():
    """Every entry point's argument list in the binding against its prototype: the same count,
    pointers where the header has pointers, and the exact scalar type and width elsewhere."""
    protos = _prototypes()
    assert set(protos) == set(_native._SIGNATURES)
    for name, (ret, args) in protos.items():
        argtypes, restype = _native._SIGNATURES[name]
        assert len(argtypes) == len(args), name
        for c_arg, py in zip(args, argtypes):
            if "*" in c_arg:
                assert _is_pointer_type(py), (name, c_arg, py)
            else:
                base = c_arg.replace("const ", "").split()[0]
                assert py is _SCALARS[base], (name, c_arg, py)
        if "*" in ret:
            assert _is_pointer_type(restype), (name, ret)
        else:
            assert restype is _SCALARS[ret.replace("const ", "")], (name, ret, restype)
