"""Builds libcube_awq.so (sm_100a) in-tree with nvcc.

    python -m cube_awq_b200.build [--force] [--verbose]

It also builds _cawq_torch.so (csrc/cawq_torch.cpp, against torch's headers
with the host compiler), the compiled host path of the module forward.

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


EXT_SRC = os.path.join(CSRC, "cawq_torch.cpp")
EXT_PATH = os.path.join(PKG_DIR, "_cawq_torch.so")


def build_torch_ext(force: bool = False, verbose: bool = False) -> str:
    """Compile _cawq_torch.so, the compiled host path of the module forward
    (a torch binding over libcube_awq.so; see csrc/cawq_torch.cpp)."""
    import sysconfig

    import torch
    from torch.utils import cpp_extension as ce
    deps = [EXT_SRC, os.path.join(INCLUDE, "cube_awq.h")]
    if not force and not _stale(EXT_PATH, deps):
        return EXT_PATH
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    torch_lib = os.path.join(os.path.dirname(torch.__file__), "lib")
    inc = ce.include_paths(device_type="cuda") + [sysconfig.get_paths()["include"], INCLUDE]
    cxx = "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else "g++"
    tmp = EXT_PATH + ".tmp"
    cmd = [cxx, "-O2", "-std=c++17", "-shared", "-fPIC", "-fvisibility=hidden",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=_cawq_torch",
           "-DTORCH_API_INCLUDE_EXTENSION_H"] + [f"-I{d}" for d in inc] + [
           EXT_SRC, "-o", tmp, f"-L{torch_lib}", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu",
           "-ltorch_python", f"-L{PKG_DIR}", "-lcube_awq", "-Wl,-rpath,$ORIGIN",
           f"-Wl,-rpath,{torch_lib}"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"torch extension build failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, EXT_PATH)
    return EXT_PATH


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers / spills / smem")
    a = ap.parse_args(argv)
    print(build(force=a.force, verbose=a.verbose, ptxas_info=a.ptxas_info))
    print(build_torch_ext(force=a.force, verbose=a.verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
