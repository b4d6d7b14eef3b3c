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
TORCH_LIB = PKG / "libkvr_torch.so"
SOURCES = ["kvr_capi.cu", "kvr_pack.cu", "kvr_decode.cu", "kvr_decode_simt.cu", "kvr_exchange.cu"]
TORCH_SOURCE = "kvr_torch.cpp"
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
    """Compile libkvr.so and the torch operator library; returns libkvr.so's path."""
    lib = build_lib(force, verbose, ptxas_info)
    build_torch_ops(force, verbose)
    return lib


def _torch_stale() -> bool:
    if not TORCH_LIB.exists():
        return True
    mtime = TORCH_LIB.stat().st_mtime
    deps = [CSRC / TORCH_SOURCE, ROOT / "include" / "kvr.h", LIB]
    return any(p.stat().st_mtime > mtime for p in deps if p.exists())


def build_torch_ops(force: bool = False, verbose: bool = False) -> Path:
    """libkvr_torch.so: the torch.ops.kvr operators (kvr_torch.cpp, host C++
    over libkvr.so's C ABI), compiled against this interpreter's torch."""
    if not force and not _torch_stale():
        return TORCH_LIB
    import torch
    from torch.utils import cpp_extension

    cxx = host_cxx()
    cuda_home = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = [cxx, "-O2", "-std=c++17", "-shared", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_EXTENSION_NAME=kvr_torch"]
    for inc in cpp_extension.include_paths():
        cmd += ["-isystem", inc]
    cmd += ["-isystem", str(cuda_home / "include"), "-I", str(ROOT / "include"), str(CSRC / TORCH_SOURCE)]
    for libdir in cpp_extension.library_paths():
        cmd += ["-L", libdir, f"-Wl,-rpath,{libdir}"]
    cmd += ["-L", str(PKG), "-lkvr", "-Wl,-rpath,$ORIGIN", "-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch",
            "-L", str(cuda_home / "lib64"), "-lcudart"]
    tmp = TORCH_LIB.with_suffix(".so.tmp")
    cmd += ["-o", str(tmp)]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"building {TORCH_LIB.name} failed:\n{res.stdout}\n{res.stderr}")
    _check_shared_cxx_runtime(tmp)
    os.replace(tmp, TORCH_LIB)
    return TORCH_LIB


def host_cxx() -> str:
    """The C++ compiler for the torch operator library: KVR_CXX if set, else
    the system g++.  $CXX is not used, because a compiler wrapper that links
    libstdc++ statically would give the library its own C++ runtime: a
    TORCH_CHECK exception thrown there is then caught by torch's runtime and
    the process crashes."""
    for cand in (os.environ.get("KVR_CXX"), "/usr/bin/g++", shutil.which("g++")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("g++ not found; set KVR_CXX to the C++ compiler torch was built with")


def _check_shared_cxx_runtime(lib: Path) -> None:
    """The operator library must use the shared libstdc++ that torch uses
    (see host_cxx)."""
    res = subprocess.run(["readelf", "-d", str(lib)], capture_output=True, text=True)
    if res.returncode == 0 and "libstdc++.so" not in res.stdout:
        raise RuntimeError(f"{lib.name} does not link the shared libstdc++ (statically linked C++ runtime); "
                           "build it with the system g++ (KVR_CXX)")


def build_lib(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    """Compile every CUDA source into libkvr.so; returns its path."""
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
