"""Build the sm_100a shared library ``libhyb200.so`` in-tree with nvcc.

The library holds every CUDA kernel of the package behind the C ABI declared in
``include/hyb200.h``.  It is compiled for ``sm_100a`` only (tcgen05, TMA), without
fast-math so the quantiser's IEEE divisions stay bit-exact.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
LIB_PATH = PKG_DIR / "libhyb200.so"
SOURCES = ["hyb_capi.cu", "hyb_kv.cu", "hyb_attn.cu", "hyb_comm.cu"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def _stale() -> bool:
    if not LIB_PATH.exists():
        return True
    built = LIB_PATH.stat().st_mtime
    deps = list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + [REPO_DIR / "include" / "hyb200.h"]
    return any(p.stat().st_mtime > built for p in deps)


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    """Compile (if stale) and return the path of the shared library."""
    if not force and not _stale():
        return LIB_PATH
    nvcc = nvcc_path()
    build_dir = PKG_DIR / "_build"
    build_dir.mkdir(exist_ok=True)
    common = [nvcc, "-std=c++17", "-O3", "-lineinfo", *ARCH_FLAGS, "-Xcompiler", "-fPIC",
              "-I", str(REPO_DIR / "include"), "--expt-relaxed-constexpr"]
    if ptxas_verbose:
        common += ["-Xptxas", "-v"]
    objs = []
    for src in SOURCES:
        obj = build_dir / (Path(src).stem + ".o")
        cmd = common + ["-c", str(CSRC / src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{res.stdout}\n{res.stderr}")
        if ptxas_verbose:
            print(res.stderr, file=sys.stderr)
        objs.append(str(obj))
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc, "-shared", *ARCH_FLAGS, "-o", str(tmp), *objs]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_verbose="-v" in sys.argv)
    print(LIB_PATH)
