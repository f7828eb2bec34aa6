"""Builds libcube_awq.so (sm_100a) in-tree with nvcc.

    python -m cube_awq_b200.build [--force] [--verbose]

Each translation unit under csrc/ is compiled to an object in csrc/_build/
(in parallel), then linked with the static CUDA runtime into
cube_awq_b200/libcube_awq.so. Only the extern "C" symbols of include/cube_awq.h
are exported.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG_DIR, "csrc")
BUILD_DIR = os.path.join(CSRC, "_build")
REPO = os.path.dirname(PKG_DIR)
INCLUDE = os.path.join(REPO, "include")
LIB_PATH = os.path.join(PKG_DIR, "libcube_awq.so")

SOURCES = ["cawq_api.cu", "cawq_kernels.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("CUDA_HOME", ""), "/usr/local/cuda"):
        p = os.path.join(cand, "bin", "nvcc") if cand else ""
        if p and os.path.exists(p):
            return p
    p = shutil.which("nvcc")
    if not p:
        raise RuntimeError("nvcc not found")
    return p


def _host_compiler_flags() -> list[str]:
    # Prefer the system g++ (the image's $CXX wrapper lacks some runtime bits).
    for cxx in ("/usr/bin/g++",):
        if os.path.exists(cxx):
            return ["-ccbin", cxx]
    return []


def common_flags() -> list[str]:
    return ARCH + _host_compiler_flags() + [
        "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
        "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
        "-I", INCLUDE, "-I", CSRC,
    ]


def _deps() -> list[str]:
    out = []
    for d in (CSRC, INCLUDE):
        for f in os.listdir(d):
            if f.endswith((".cu", ".cuh", ".h")):
                out.append(os.path.join(d, f))
    return out


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, verbose: bool, extra: list[str]) -> str:
    obj = os.path.join(BUILD_DIR, os.path.splitext(src)[0] + ".o")
    cmd = [nvcc()] + common_flags() + extra + ["-c", os.path.join(CSRC, src), "-o", obj]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if verbose and (r.stdout or r.stderr):
        print(r.stdout + r.stderr, flush=True)
    return obj


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> str:
    """Compile and link libcube_awq.so; returns its path."""
    os.makedirs(BUILD_DIR, exist_ok=True)
    deps = _deps()
    if not force and not _stale(LIB_PATH, deps):
        return LIB_PATH
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    with cf.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose or ptxas_info, extra), SOURCES))
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc()] + ARCH + _host_compiler_flags() + [
        "-shared", "-cudart", "static", "-o", tmp] + objs + ["-ldl", "-lpthread", "-lrt"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers / spills / smem")
    a = ap.parse_args(argv)
    print(build(force=a.force, verbose=a.verbose, ptxas_info=a.ptxas_info))
    return 0


if __name__ == "__main__":
    sys.exit(main())
