"""Build libkvr.so (the C-ABI library) in-tree with nvcc for sm_100a.

The library is plain CUDA C++ with an ``extern "C"`` surface (include/kvr.h);
it links only the CUDA runtime, so any FFI can bind it.  Never add
--use_fast_math: the quantizer's bit-exactness relies on IEEE division and
round-half-even.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libkvr.so"
SOURCES = ["kvr_capi.cu", "kvr_pack.cu", "kvr_decode.cu", "kvr_decode_simt.cu", "kvr_exchange.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; install the CUDA toolkit to build libkvr.so")


def _stale() -> bool:
    if not LIB.exists():
        return True
    mtime = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.cuh")) + [ROOT / "include" / "kvr.h"]
    return any(p.stat().st_mtime > mtime for p in deps if p.exists())


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    """Compile every source into one shared object; returns its path."""
    if not force and not _stale():
        return LIB
    nvcc = nvcc_path()
    build_dir = PKG / "_build"
    build_dir.mkdir(exist_ok=True)
    objs = []
    common = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
                     "-I", str(ROOT / "include")]
    if ptxas_info:
        common += ["-Xptxas", "-v"]
    for src in SOURCES:
        obj = build_dir / (Path(src).stem + ".o")
        cmd = [nvcc, *common, "-c", str(CSRC / src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{res.stdout}\n{res.stderr}")
        if ptxas_info or verbose:
            sys.stderr.write(res.stderr)
        objs.append(str(obj))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH, "-shared", "-o", str(tmp), *objs, "-lcudart"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_info="--ptxas" in sys.argv)
    print(LIB)
