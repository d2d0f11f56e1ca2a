"""Build librtgs2d.so (all CUDA sources, sm_100a) in-tree with nvcc.

The library is written next to this file under ``_lib/`` so that it travels with the source
tree; nothing is installed into site-packages.
"""

from __future__ import annotations

import concurrent.futures
import os
import shutil
import subprocess
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR.parent / "csrc"
INCLUDE = PKG_DIR.parents[1] / "include"
LIB_DIR = PKG_DIR / "_lib"
LIB_PATH = LIB_DIR / "librtgs2d.so"
SOURCES = ("capi.cu", "project.cu", "binning.cu", "raster.cu", "optim.cu", "fit_engine.cu", "noalloc.cu", "sort.cu")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-ffp-contract=off",
    "-Xcompiler", "-fvisibility=hidden",
]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(cuda_home) / "bin" / "nvcc"
    if cand.exists():
        return str(cand)
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found: set CUDA_HOME or put nvcc on PATH")
    return found


def _stale() -> bool:
    if not LIB_PATH.exists():
        return True
    lib_mtime = LIB_PATH.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh"))
    deps += list(INCLUDE.glob("*.h"))
    return any(p.stat().st_mtime > lib_mtime for p in deps)


def build_library(force: bool = False, verbose: bool = False) -> Path:
    """Compile and link librtgs2d.so for sm_100a; returns its path. Skips if up to date."""
    if not force and not _stale():
        return LIB_PATH
    nvcc = _nvcc()
    obj_dir = LIB_DIR / "obj"
    obj_dir.mkdir(parents=True, exist_ok=True)

    def compile_one(src: str) -> Path:
        obj = obj_dir / (Path(src).stem + ".o")
        cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, "-I", str(INCLUDE), "-c", str(CSRC / src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd))
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{res.stdout}\n{res.stderr}")
        return obj

    with concurrent.futures.ThreadPoolExecutor(max_workers=len(SOURCES)) as pool:
        objs = list(pool.map(compile_one, SOURCES))
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    import sys

    print(build_library(force="--force" in sys.argv, verbose="-v" in sys.argv))
