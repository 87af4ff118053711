"""Builds the B200 operator library and its C++ host layer.

  lib/libhc_b200.so    : csrc/*.cu compiled with nvcc for sm_100a -- the C-ABI (include/*.h)
  lib/libhc_harness.so : host/src/*.cpp compiled with g++ -- the harness::device runtime and the
                         per-op C++ runners (host/include/harness/*.hpp), linked to libhc_b200.so

Usage: python build.py [--force] [--verbose]

Each translation unit is compiled to an object in parallel (only when its sources changed),
then linked into one shared library.  ptxas resource usage (-Xptxas -v) is written to
lib/ptxas_<unit>.log for register / spill / shared-memory review.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
LIB = HERE / "lib"
INCLUDE = ROOT / "include"
TARGET = LIB / "libhc_b200.so"
HOST = HERE / "host"
HOST_TARGET = LIB / "libhc_harness.so"
HOST_FLAGS = ["-O2", "-std=c++17", "-fPIC", "-Wall", "-Wextra", f"-I{INCLUDE}", f"-I{HOST / 'include'}"]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
                "--expt-relaxed-constexpr", f"-I{INCLUDE}", f"-I{CSRC}"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found (needs the CUDA toolkit)")
    return cand


def _deps(src: Path) -> list[Path]:
    return [src] + sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _stale(out: Path, deps: list[Path]) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path, verbose: bool) -> Path:
    obj = LIB / "obj" / (src.stem + ".o")
    obj.parent.mkdir(parents=True, exist_ok=True)
    log = LIB / f"ptxas_{src.stem}.log"
    cmd = [nvcc(), *ARCH_FLAGS, *COMMON_FLAGS, "-Xptxas", "-v", "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    log.write_text(r.stdout + r.stderr)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stderr[-6000:]}")
    return obj


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compiles every csrc/*.cu for sm_100a and links lib/libhc_b200.so; returns its path."""
    LIB.mkdir(parents=True, exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    todo = [s for s in sources if force or _stale(LIB / "obj" / (s.stem + ".o"), _deps(s))]
    if todo:
        workers = min(len(todo), os.cpu_count() or 4)
        with cf.ThreadPoolExecutor(max_workers=workers) as ex:
            list(ex.map(lambda s: _compile(s, verbose), todo))
    objs = [LIB / "obj" / (s.stem + ".o") for s in sources]
    if force or todo or _stale(TARGET, objs):
        cmd = [nvcc(), *ARCH_FLAGS, "-shared", "-Xcompiler", "-fPIC", *map(str, objs), "-o", str(TARGET)]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr[-6000:]}")
    build_host(force, verbose)
    return TARGET


def build_host(force: bool = False, verbose: bool = False) -> Path:
    """Compiles the C++ host layer (host/src/*.cpp) into lib/libhc_harness.so, linked to libhc_b200.so."""
    srcs = sorted((HOST / "src").glob("*.cpp"))
    deps = srcs + sorted((HOST / "include").rglob("*.hpp")) + sorted(INCLUDE.glob("*.h")) + [TARGET]
    if not force and not _stale(HOST_TARGET, deps):
        return HOST_TARGET
    cxx = shutil.which("g++") or "g++"
    cmd = [cxx, *HOST_FLAGS, "-shared", *map(str, srcs), "-o", str(HOST_TARGET), f"-L{LIB}", "-lhc_b200",
           "-Wl,-rpath,$ORIGIN"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"host layer build failed:\n{r.stderr[-6000:]}")
    return HOST_TARGET


TORCH_TARGET = LIB / "libhc_torch.so"


def build_torch(force: bool = False, verbose: bool = False) -> Path:
    """Compiles csrc/torch_ops.cpp (the `hc` torch custom-op library over the C ABI) into lib/libhc_torch.so,
    linked to libhc_b200.so.  Load it with torch.ops.load_library()."""
    src = CSRC / "torch_ops.cpp"
    deps = [src, TARGET] + sorted(INCLUDE.glob("*.h"))
    if not force and not _stale(TORCH_TARGET, deps):
        return TORCH_TARGET
    import torch
    from torch.utils import cpp_extension as ce

    cxx = shutil.which("g++") or "g++"
    cmd = [cxx, "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}",
           *[f"-I{p}" for p in ce.include_paths(device_type="cuda")], f"-I{INCLUDE}", str(src), "-o", str(TORCH_TARGET),
           *[f"-L{p}" for p in ce.library_paths(device_type="cuda")], "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu",
           "-ltorch_cuda", f"-L{LIB}", "-lhc_b200", "-Wl,-rpath,$ORIGIN"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"torch op library build failed:\n{r.stderr[-6000:]}")
    return TORCH_TARGET


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    try:
        print(build(a.force, a.verbose))
        print(build_torch(a.force, a.verbose))
    except RuntimeError as e:
        print(e, file=sys.stderr)
        sys.exit(1)
