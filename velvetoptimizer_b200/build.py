"""Build ``libvesper_moe.so`` (the C-ABI library and its sm_100a kernels) in-tree.

    python -m velvetoptimizer_b200.build [--force] [--verbose]

Each ``csrc/*.cu`` is compiled by nvcc for ``sm_100a`` into ``_build/`` in parallel and
linked into ``velvetoptimizer_b200/lib/libvesper_moe.so``.  The CUDA runtime is linked
statically; kernels launch on the caller's stream.  nvcc cross-compiles, so this runs on
a machine without a GPU.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(REPO, "_build")
LIB_DIR = os.path.join(PKG, "lib")
LIB = os.path.join(LIB_DIR, "libvesper_moe.so")
INCLUDE = os.path.join(REPO, "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3,-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-I", INCLUDE, "-I", CSRC]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: set NVCC or install the CUDA toolkit")


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps() -> list[str]:
    return sources() + glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) \
        + glob.glob(os.path.join(INCLUDE, "*.h"))


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(p) <= t for p in _deps())


def _compile(src: str, verbose: bool, extra: list[str]) -> str:
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    cmd = [nvcc(), *ARCH, *FLAGS, *extra, "-c", src, "-o", obj]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
    if verbose and (r.stdout or r.stderr):
        print(r.stdout + r.stderr, flush=True)
    return obj


PARAM_KEY_SRC = os.path.join(PKG, "csrc_py", "param_key.cpp")
PARAM_KEY_LIB = os.path.join(LIB_DIR, "_param_key.so")


def build_param_key(force: bool = False, verbose: bool = False) -> str:
    """The modules' host helper (csrc_py/param_key.cpp, a CPython extension against torch's
    headers): g++ only, no GPU code.  Skips work when up to date."""
    if (not force and os.path.exists(PARAM_KEY_LIB)
            and os.path.getmtime(PARAM_KEY_SRC) <= os.path.getmtime(PARAM_KEY_LIB)):
        return PARAM_KEY_LIB
    import sysconfig

    import torch
    tdir = os.path.dirname(torch.__file__)
    abi = int(getattr(torch._C, "_GLIBCXX_USE_CXX11_ABI", True))
    cmd = [os.environ.get("CXX", "g++"), "-O2", "-std=c++17", "-fPIC", "-shared",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-I", sysconfig.get_paths()["include"],
           "-I", os.path.join(tdir, "include"),
           "-I", os.path.join(tdir, "include", "torch", "csrc", "api", "include"),
           PARAM_KEY_SRC, "-o", PARAM_KEY_LIB + ".tmp", "-L", os.path.join(tdir, "lib"),
           "-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python",
           f"-Wl,-rpath,{os.path.join(tdir, 'lib')}"]
    os.makedirs(LIB_DIR, exist_ok=True)
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"param_key build failed:\n{r.stdout}\n{r.stderr}")
    os.replace(PARAM_KEY_LIB + ".tmp", PARAM_KEY_LIB)
    return PARAM_KEY_LIB


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> str:
    """Compile and link the library (and the modules' host helper); returns the library's
    path.  Skips work when up to date."""
    build_param_key(force=force, verbose=verbose)
    if not force and not extra and up_to_date():
        return LIB
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    srcs = sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose, extra or []), srcs))
    tmp = LIB + ".tmp"
    cmd = [nvcc(), *ARCH, "-shared", "-o", tmp, *objs, "-Xcompiler", "-fPIC"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    force = "--force" in sys.argv
    verbose = "--verbose" in sys.argv or "-v" in sys.argv
    extra = ["-Xptxas", "-v"] if "--ptxas" in sys.argv else None
    print(build(force=force or bool(extra), verbose=verbose or bool(extra), extra=extra))
