"""Build recipe for the package's native code, in-tree.

  libmgb200.so   the C ABI (include/metagross_b200.h) over the sm_100a kernels
                 in csrc/*.cu, compiled with nvcc for compute_100a/sm_100a
  _C.<abi>.so    the torch extension exposing the reference's op surface; it
                 links libmgb200.so (rpath $ORIGIN) and contains no kernels

Both land next to this file, so they travel with the working tree.  Nothing is
JIT-compiled at import time: a missing library is an error, never a fallback.

    python -m metagross_b200.build [--force] [-j N]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys
import sysconfig

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(PKG, "_build")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
LIB = os.path.join(PKG, "libmgb200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
              "--expt-relaxed-constexpr"]


def ext_suffix() -> str:
    return sysconfig.get_config_var("EXT_SUFFIX") or ".so"


def ext_path() -> str:
    return os.path.join(PKG, "_C" + ext_suffix())


def _newer(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"build step failed ({r.returncode}):\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return r


def build_lib(force=False, jobs=8, verbose=False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    cus = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = sorted(glob.glob(os.path.join(CSRC, "*.cuh"))) + [os.path.join(INCLUDE, "metagross_b200.h")]
    objs = []
    todo = []
    for cu in cus:
        obj = os.path.join(BUILD, os.path.basename(cu)[:-3] + ".o")
        objs.append(obj)
        if force or _newer(obj, [cu] + headers):
            todo.append([NVCC, *ARCH, *NVCC_FLAGS, "-I", INCLUDE, "-I", CSRC, "-c", cu, "-o", obj])
    with cf.ThreadPoolExecutor(max_workers=max(1, jobs)) as ex:
        list(ex.map(lambda c: _run(c, verbose), todo))
    if force or todo or _newer(LIB, objs):
        _run([NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-Xcompiler", "-fPIC"], verbose)
    return LIB


def build_ext(force=False, verbose=False) -> str:
    import torch
    from torch.utils import cpp_extension as ce

    out = ext_path()
    src = os.path.join(CSRC, "bindings.cpp")
    deps = [src, os.path.join(INCLUDE, "metagross_b200.h"), LIB]
    if not (force or _newer(out, deps)):
        return out
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    inc = []
    for p in ce.include_paths():
        inc += ["-isystem", p]
    inc += ["-isystem", os.path.join(CUDA_HOME, "include"), "-isystem", sysconfig.get_paths()["include"]]
    libdirs = []
    for p in ce.library_paths():
        libdirs += ["-L", p, f"-Wl,-rpath,{p}"]
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_API_INCLUDE_EXTENSION_H", "-DTORCH_EXTENSION_NAME=_C", *inc, "-I", INCLUDE, src, "-o", out,
           *libdirs, "-L", PKG, "-lmgb200", "-Wl,-rpath,$ORIGIN", "-lc10", "-ltorch", "-ltorch_cpu",
           "-ltorch_python", "-lc10_cuda", "-ltorch_cuda"]
    _run(cmd, verbose)
    return out


def build(force=False, jobs=8, verbose=False):
    build_lib(force=force, jobs=jobs, verbose=verbose)
    build_ext(force=force, verbose=verbose)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=8)
    ap.add_argument("-v", action="store_true")
    a = ap.parse_args()
    build(force=a.force, jobs=a.j, verbose=a.v)
    print("built", LIB, ext_path(), file=sys.stderr)
