"""Builds libhs_ext.so in-tree with nvcc for sm_100a.

The library is a plain C-ABI shared object (no torch headers), so the same
binary serves the Python host layer (ctypes) and any other FFI a reference
maintainer would bind. The built file lives next to this module so it travels
with the source tree to the GPU host.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
INCLUDE = PKG_DIR.parent / "include"
LIB_PATH = PKG_DIR / "libhs_ext.so"
TRACE_LIB_PATH = PKG_DIR / "libhs_ext_trace.so"  # the same sources with -DHS_TRACE (trace.py)
SOURCES = ["hs_util.cu", "hs_router.cu", "hs_moe.cu", "hs_accept.cu", "hs_norm.cu", "hs_head.cu", "hs_state.cu", "hs_ep.cu"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the CUDA 12.9 toolkit is required to build libhs_ext.so")
    return cand


def _inputs() -> list[Path]:
    return [CSRC / s for s in SOURCES] + list(CSRC.glob("*.cuh")) + [INCLUDE / "hs_ext.h"]


def is_stale(lib: Path = LIB_PATH) -> bool:
    if not lib.exists():
        return True
    t = lib.stat().st_mtime
    return any(p.stat().st_mtime > t for p in _inputs())


def build(force: bool = False, verbose: bool = False, trace: bool = False) -> Path:
    """Compile every CUDA source into one shared library (idempotent). trace:
    the tracing build (-DHS_TRACE: the layer call's kernels stamp their phase
    boundaries, read by home_seek_b200/trace.py) into libhs_ext_trace.so."""
    lib = TRACE_LIB_PATH if trace else LIB_PATH
    if not force and not is_stale(lib):
        return lib
    out_dir = PKG_DIR / ("_build_trace" if trace else "_build")
    out_dir.mkdir(exist_ok=True)
    nvcc = _nvcc()
    common = ARCH_FLAGS + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I", str(INCLUDE),
                           "--expt-relaxed-constexpr"] + (["-DHS_TRACE"] if trace else [])
    if verbose:
        common += ["-Xptxas", "-v"]
    objs = []
    for s in SOURCES:
        obj = out_dir / (Path(s).stem + ".o")
        cmd = [nvcc, "-c", str(CSRC / s), "-o", str(obj)] + common
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0 or verbose:
            sys.stderr.write(r.stdout + r.stderr)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {s}")
        objs.append(str(obj))
    tmp = lib.with_suffix(".so.tmp")
    cmd = [nvcc, "-shared", "-o", str(tmp)] + [str(o) for o in objs] + ARCH_FLAGS + ["-Xcompiler", "-fPIC", "-ldl"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc link failed")
    os.replace(tmp, lib)
    return lib


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv, trace="--trace" in sys.argv))
