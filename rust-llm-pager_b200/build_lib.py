"""Build the two C-ABI libraries of this package.

``libpager_b200.so``: the decode-attention library for sm_100a.  Every
``csrc/*.cu`` is compiled to an object with nvcc in parallel and linked next to
this file.  nvcc cross-compiles: no GPU is needed.

``libpager_core.so``: the block-placement pager (``csrc/pager_core.cpp``), host
code only, built with the host C++ compiler and ``-ffp-contract=off`` so that
its f32 score arithmetic rounds after every operation.

    python rust-llm-pager_b200/build_lib.py [--force] [--verbose]
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libpager_b200.so")
CORE_LIB = os.path.join(HERE, "libpager_core.so")
CXX = os.environ.get("CXX", "g++")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", f"-I{INCLUDE}", f"-I{CSRC}"]


def _sources():
    return sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))


def _headers_mtime():
    files = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    files += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    return max(os.path.getmtime(f) for f in files)


def _compile(src, force, verbose):
    obj = os.path.join(BUILD, src.replace(".cu", ".o"))
    srcp = os.path.join(CSRC, src)
    if not force and os.path.exists(obj):
        if os.path.getmtime(obj) >= max(os.path.getmtime(srcp), _headers_mtime()):
            return obj, ""
    cmd = [NVCC] + FLAGS + (["-Xptxas", "-v"] if verbose else []) + ["-c", srcp, "-o", obj]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{res.stderr}")
    return obj, res.stderr


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        results = list(ex.map(lambda s: _compile(s, force, verbose), srcs))
    objs = [o for o, _ in results]
    if verbose:
        for (o, log) in results:
            if log:
                sys.stderr.write(f"--- {os.path.basename(o)}\n{log}")
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cmd = [NVCC] + ARCH + ["-shared", "-o", LIB] + objs
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stderr}")
    build_core(force)
    return LIB


def build_core(force: bool = False) -> str:
    src = os.path.join(CSRC, "pager_core.cpp")
    hdr = os.path.join(INCLUDE, "pager_core.h")
    if not force and os.path.exists(CORE_LIB) and os.path.getmtime(CORE_LIB) >= max(
            os.path.getmtime(src), os.path.getmtime(hdr)):
        return CORE_LIB
    cmd = [CXX, "-O2", "-std=c++17", "-fPIC", "-shared", "-ffp-contract=off", "-fvisibility=hidden", "-Wl,--exclude-libs,ALL", "-Wall", "-Wextra", f"-I{INCLUDE}",
           src, "-o", CORE_LIB]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"{CXX} failed for pager_core.cpp:\n{res.stderr}")
    return CORE_LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
