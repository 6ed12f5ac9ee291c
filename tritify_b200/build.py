"""Build tritify_b200/libktmoe.so: the sm_100a kernels and the C ABI of include/ktmoe.h.

nvcc cross-compiles for sm_100a without a GPU, so this runs anywhere the CUDA toolkit is installed. The library is
built in-tree so it travels with the repository to the GPU host.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libktmoe.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
SOURCES_CU = ["ktmoe.cu", "noalloc.cu"]
SOURCES_CPP = ["host_prep.cpp", "wire.cpp"]
HEADERS = ["fixed_point.cuh", "digit_gemm.cuh", "digit_gemm_pair.cuh", "moe_kernels.cuh", "ep_peer.cuh", "synth.cuh",
           "host_prep.h"]


def _nvcc() -> str:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libktmoe.so")


def _nccl() -> tuple[list[str], list[str]]:
    """Compile and link flags for NCCL. The library uses the NCCL that PyTorch loads (the nvidia-nccl wheel) when it
    is installed, so that a process importing both sees one NCCL: with two, whichever loads first provides the
    symbols and the other library can fail to import. Otherwise the system NCCL."""
    import importlib.util

    spec = importlib.util.find_spec("nvidia.nccl")
    if spec and spec.submodule_search_locations:
        base = list(spec.submodule_search_locations)[0]
        lib, inc = os.path.join(base, "lib"), os.path.join(base, "include")
        if os.path.exists(os.path.join(lib, "libnccl.so.2")) and os.path.exists(os.path.join(inc, "nccl.h")):
            return ["-I", inc], ["-L", lib, "-l:libnccl.so.2", "-Xlinker", "-rpath," + lib]
    return [], ["-lnccl"]


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile (if stale) and return the path of libktmoe.so."""
    os.makedirs(BUILD, exist_ok=True)
    nvcc = _nvcc()
    header_deps = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(ROOT, "include", "ktmoe.h")]
    nccl_inc, nccl_link = _nccl()
    objs = []
    for src in SOURCES_CPP:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src + ".o")
        objs.append(o)
        if force or _stale(o, [s] + header_deps):
            cmd = ["g++", "-O3", "-std=c++17", "-fPIC", "-ffp-contract=off", "-Wall", "-I", os.path.join(ROOT, "include"),
                   "-c", s, "-o", o]
            _run(cmd, verbose)
    for src in SOURCES_CU:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src + ".o")
        objs.append(o)
        if force or _stale(o, [s] + header_deps):
            cmd = [nvcc, *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC,-ffp-contract=off",
                   "-I", os.path.join(ROOT, "include"), "-I", CSRC, *nccl_inc, "-c", s, "-o", o]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
            _run(cmd, verbose)
    if force or _stale(LIB, objs):
        _run([nvcc, *ARCH, "-shared", "-o", LIB, *objs, *nccl_link, "-lpthread"], verbose)
    return LIB


def _run(cmd: list[str], verbose: bool) -> None:
    cmd = [c for c in cmd if c]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {' '.join(cmd[:3])} ...")
    if verbose and (r.stdout or r.stderr):
        sys.stderr.write(r.stdout + r.stderr)


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
