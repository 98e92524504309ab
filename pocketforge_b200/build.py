"""Builds pocketforge_b200/libpf_b200.so for sm_100a (nvcc cross-compiles; no GPU needed).

    python -m pocketforge_b200.build [--force]

Objects go to pocketforge_b200/_build/ (git-ignored); the shared library is
written next to this file so that it travels with the source tree.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libpf_b200.so")
FORGE = os.path.join(HERE, "forge")  # the forge:: C++ API over the C ABI
FORGE_LIB = os.path.join(HERE, "libforge_b200.so")  # the same library under the name forge:: users link
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
              "-Xcompiler", "-fvisibility=hidden", "-I" + INCLUDE]
CXX_FLAGS = ["-O2", "-std=c++17", "-fPIC", "-fvisibility=hidden", "-I" + INCLUDE]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return cand


def sources():
    cu = sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))
    cpp = sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cpp"))
    cpp += sorted(os.path.join(FORGE, f) for f in os.listdir(FORGE) if f.endswith(".cpp"))
    return cu, cpp


def _deps_mtime(src: str) -> float:
    m = os.path.getmtime(src)
    for d in (CSRC, FORGE):
        for f in os.listdir(d):
            if f.endswith((".cuh", ".h", ".hpp")):
                m = max(m, os.path.getmtime(os.path.join(d, f)))
    for root, _, files in os.walk(INCLUDE):
        for f in files:
            m = max(m, os.path.getmtime(os.path.join(root, f)))
    return m


def _compile(path: str, force: bool) -> str:
    src = os.path.relpath(path, HERE).replace(os.sep, "_")
    obj = os.path.join(BUILD, src + ".o")
    if not force and os.path.exists(obj) and os.path.getmtime(obj) >= _deps_mtime(path):
        return obj
    if src.endswith(".cu"):
        cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", path, "-o", obj]
    else:
        cmd = [os.environ.get("CXX", "g++"), *CXX_FLAGS, "-I/usr/local/cuda/include", "-c", path, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return obj


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    cu, cpp = sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force), cu + cpp))
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", LIB, *objs, "-lcudart_static", "-lrt", "-lpthread", "-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    if not os.path.islink(FORGE_LIB):
        if os.path.exists(FORGE_LIB):
            os.remove(FORGE_LIB)
        os.symlink(os.path.basename(LIB), FORGE_LIB)
    if verbose:
        print(LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
