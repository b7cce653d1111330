"""Builds libwhistle_b200.so in-tree with nvcc for sm_100a (no GPU needed),
and the C++ host mirror libwhistle_b200_host.so (g++) beside it.

    python go-whistle_b200/build.py [--verbose]

Every ``csrc/*.cu`` is compiled to an object with
``-gencode arch=compute_100a,code=sm_100a`` and linked into one shared
library beside this file. The CUDA runtime is linked statically, so the
library needs only the driver at run time.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
LIB = HERE / "libwhistle_b200.so"
HOST = HERE / "host"
HOST_LIB = HERE / "libwhistle_b200_host.so"
OBJ = HERE / "_build"
INCLUDE = HERE.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVFLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
           "-I", str(INCLUDE)]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA library cannot be built")


def sources():
    return sorted(CSRC.glob("*.cu"))


def _stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + [INCLUDE / "whistle_b200.h", Path(__file__)]
    return any(d.stat().st_mtime > t for d in deps)


def _host_stale() -> bool:
    if not HOST_LIB.exists():
        return True
    t = HOST_LIB.stat().st_mtime
    deps = list(HOST.glob("*.cpp")) + list(HOST.glob("*.hpp")) + [LIB, INCLUDE / "whistle_b200.h"]
    return any(d.stat().st_mtime > t for d in deps)


def build_host(force: bool = False, verbose: bool = False) -> Path:
    """The C++ host mirror (host/whistle.hpp) as libwhistle_b200_host.so,
    linked against libwhistle_b200.so beside it."""
    if not force and not _host_stale():
        return HOST_LIB
    cxx = os.environ.get("CXX") or shutil.which("g++") or "g++"
    tmp = HOST_LIB.with_suffix(".so.tmp")
    cmd = [cxx, "-O2", "-std=c++17", "-Wall", "-Wextra", "-fPIC", "-shared", "-I", str(INCLUDE),
           *map(str, sorted(HOST.glob("*.cpp"))), "-o", str(tmp), "-L", str(HERE), "-lwhistle_b200",
           "-Wl,-rpath,$ORIGIN"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
    if r.returncode != 0:
        raise RuntimeError("g++ failed on the C++ host mirror")
    os.replace(tmp, HOST_LIB)
    return HOST_LIB


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not _stale():
        build_host(force=False, verbose=verbose)
        return LIB
    OBJ.mkdir(exist_ok=True)
    cc = nvcc()
    objs = []
    for src in sources():
        obj = OBJ / (src.stem + ".o")
        # The decoder's elementwise arithmetic must keep every float
        # rounding the reference makes: no multiply-add contraction there.
        extra = ["--fmad=false"] if src.name == "decoder.cu" else []
        cmd = [cc, *ARCH, *NVFLAGS, *extra, "-c", str(src), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        r = subprocess.run(cmd, capture_output=True, text=True)
        if verbose or r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}")
        objs.append(str(obj))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [cc, *ARCH, "-shared", "-o", str(tmp), *objs, "-lcudart_static", "-lrt", "-ldl",
           "-lpthread"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc link failed")
    os.replace(tmp, LIB)
    build_host(force=True, verbose=verbose)
    return LIB


if __name__ == "__main__":
    build(force=True, verbose="--verbose" in sys.argv)
    print(LIB)
