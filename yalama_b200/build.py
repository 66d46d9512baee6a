"""Build the engine library in-tree: yalama_b200/lib/libyalama_b200.so.

Every .cu file is compiled by nvcc for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``), the host files by g++, and the
result is linked against the static CUDA runtime and the NCCL that ships with
the image's torch wheel (``nvidia/nccl``). Cross-compiles without a GPU.

    python -m yalama_b200.build [--force] [--verbose]
"""
from __future__ import annotations

import argparse
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
ROOT = os.path.dirname(HERE)
OBJ = os.path.join(ROOT, "_build", "obj")
LIB_DIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIB_DIR, "libyalama_b200.so")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nccl_dirs():
    import importlib.util
    spec = importlib.util.find_spec("nvidia")
    for base in (list(spec.submodule_search_locations) if spec and spec.submodule_search_locations else []):
        inc, lib = os.path.join(base, "nccl", "include"), os.path.join(base, "nccl", "lib")
        if os.path.exists(os.path.join(inc, "nccl.h")):
            return inc, lib
    return "/usr/include", "/usr/lib/x86_64-linux-gnu"


def _stale(src_files, target):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in src_files)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("build step failed: " + " ".join(cmd[:3]) + " ...")
    return r


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    nccl_inc, nccl_lib = nccl_dirs()
    headers = glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        [os.path.join(ROOT, "include", "yalama_b200.h")]
    objs = []
    nvcc = os.path.join(CUDA, "bin", "nvcc")
    for src in sorted(glob.glob(os.path.join(CSRC, "*.cu"))):
        obj = os.path.join(OBJ, os.path.basename(src) + ".o")
        objs.append(obj)
        if force or _stale([src] + headers, obj):
            _run([nvcc, *ARCH, "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
                  "-Xptxas", "-warn-spills", "-I", CSRC, "-c", src, "-o", obj], verbose)
    for src in sorted(glob.glob(os.path.join(CSRC, "*.cpp"))):
        obj = os.path.join(OBJ, os.path.basename(src) + ".o")
        objs.append(obj)
        if force or _stale([src] + headers, obj):
            _run(["g++", "-O2", "-std=c++17", "-fPIC", "-Wall", "-Wno-unused-function",
                  "-I", CSRC, "-I", os.path.join(CUDA, "include"), "-I", nccl_inc, "-c", src, "-o", obj], verbose)
    if force or _stale(objs, LIB):
        _run(["g++", "-shared", "-o", LIB, *objs,
              "-L", os.path.join(CUDA, "lib64"), "-lcudart_static", "-ldl", "-lrt", "-lpthread",
              "-L", nccl_lib, "-l:libnccl.so.2", "-Wl,-rpath," + nccl_lib,
              "-Wl,--no-undefined"], verbose)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.verbose))


if __name__ == "__main__":
    main()
