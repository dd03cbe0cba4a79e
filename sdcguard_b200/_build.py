"""Builds the native library `sdcguard_b200/_lib/libsdcguard_b200.so` from `csrc/*.cu` and `csrc/*.cpp`, and the
host-only probe library `_lib/libsdcguard_host.so` from `csrc/host/*.cpp`.

Every CUDA source is compiled for sm_100a only (`-gencode arch=compute_100a,code=sm_100a`) with nvcc, in
parallel, into objects under `_lib/obj/`, then linked into one shared library that Python loads with ctypes
(`sdcguard_b200._native`). The library has no PyTorch dependency: it takes raw device pointers and a CUDA
stream, so the same entry points serve Python, C++ callers and tests.

    python -m sdcguard_b200._build            # incremental
    python -m sdcguard_b200._build --force    # rebuild everything
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
SRC = PKG / "csrc"
OUT = PKG / "_lib"
OBJ = OUT / "obj"
LIB = OUT / "libsdcguard_b200.so"
HOST_SRC = SRC / "host"
HOST_LIB = OUT / "libsdcguard_host.so"     # host-only C++ (cuBLAS / cuBLASLt probe), linked to the CUDA libraries

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVFLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
           "-Xcompiler", "-Wno-unused-function", "-DNDEBUG"]
CXXFLAGS = ["-O3", "-std=c++17", "-fPIC", "-Wall", "-Wno-unused-function"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def cuda_home() -> Path:
    return Path(nvcc()).resolve().parent.parent


def sources() -> list[Path]:
    return sorted(p for p in SRC.iterdir() if p.suffix in (".cu", ".cpp"))


def _headers_mtime() -> float:
    hs = [p.stat().st_mtime for p in SRC.iterdir() if p.suffix in (".cuh", ".h", ".hpp")]
    return max(hs) if hs else 0.0


def _compile(src: Path, force: bool, extra: list[str]) -> tuple[Path, str]:
    obj = OBJ / (src.name + ".o")
    if not force and obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, _headers_mtime()):
        return obj, ""
    if src.suffix == ".cu":
        cmd = [nvcc(), *ARCH, *NVFLAGS, *extra, "-I", str(SRC), "-c", str(src), "-o", str(obj)]
    else:
        cmd = ["g++", *CXXFLAGS, "-I", str(SRC), "-I", str(cuda_home() / "include"), "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compiling {src.name} failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return obj, (r.stderr or "")


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    """Compile every source (in parallel) and link the shared library. Returns the library path."""
    OBJ.mkdir(parents=True, exist_ok=True)
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []
    srcs = sources()
    with cf.ThreadPoolExecutor(max_workers=min(16, os.cpu_count() or 4)) as ex:
        results = list(ex.map(lambda s: _compile(s, force or ptxas_verbose, extra), srcs))
    objs = [o for o, _ in results]
    if verbose or ptxas_verbose:
        for (o, log), s in zip(results, srcs):
            if log:
                print(f"== {s.name}\n{log}", file=sys.stderr)
    newest = max(o.stat().st_mtime for o in objs)
    if force or not LIB.exists() or LIB.stat().st_mtime < newest:
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart_static", "-lrt", "-ldl",
               "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"linking failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


def build_host(force: bool = False) -> Path:
    """The host-only library: `csrc/host/*.cpp` with g++, linked to cuBLAS, cuBLASLt and the CUDA runtime."""
    srcs = sorted(HOST_SRC.glob("*.cpp"))
    OUT.mkdir(parents=True, exist_ok=True)
    if not force and HOST_LIB.exists() and HOST_LIB.stat().st_mtime >= max(p.stat().st_mtime for p in srcs):
        return HOST_LIB
    home = cuda_home()
    tmp = HOST_LIB.with_suffix(".so.tmp")
    cmd = ["g++", *CXXFLAGS, "-shared", "-I", str(home / "include"), *map(str, srcs), "-o", str(tmp),
           "-L", str(home / "lib64"), f"-Wl,-rpath,{home / 'lib64'}", "-lcublasLt", "-lcublas", "-lcudart"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"building the host library failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, HOST_LIB)
    return HOST_LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true", help="print registers / spills / smem per kernel")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args(argv)
    print(build(force=a.force, verbose=a.verbose, ptxas_verbose=a.ptxas_verbose))
    print(build_host(force=a.force))
    return 0


if __name__ == "__main__":
    sys.exit(main())
