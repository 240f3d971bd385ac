"""Build the sm_100a shared library ``libuttt_b200.so`` in-tree with nvcc.

    python -m utttcompanion_b200.build          # incremental
    python -m utttcompanion_b200.build --force  # rebuild everything

Each ``csrc/*.cu`` is compiled to an object under ``csrc/_build/`` and the
objects are linked into ``utttcompanion_b200/libuttt_b200.so`` (CUDA runtime
linked statically; no libcuda link: tensor maps are encoded through the
runtime's driver entry point).  Only sm_100a code is generated.
"""

from __future__ import annotations

import argparse
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(CSRC, "_build")
LIB = os.path.join(PKG, "libuttt_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--use_fast_math", "-Xptxas", "-v",
              "-Wno-deprecated-gpu-targets", "--expt-relaxed-constexpr"]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libuttt_b200.so")
    return path


def _stale(src: str, obj: str, headers) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return os.path.getmtime(src) > t or any(os.path.getmtime(h) > t for h in headers)


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = sorted(glob.glob(os.path.join(CSRC, "*.cuh"))) + [os.path.join(ROOT, "include", "uttt_b200.h")]
    objs = []
    relink = force or not os.path.exists(LIB)
    for src in sources:
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if force or _stale(src, obj, headers):
            cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-I", os.path.join(ROOT, "include"), "-c", src, "-o", obj]
            res = subprocess.run(cmd, capture_output=True, text=True)
            log = os.path.join(BUILD, os.path.basename(src) + ".log")
            with open(log, "w") as fh:
                fh.write(res.stdout + res.stderr)
            if res.returncode != 0:
                sys.stderr.write(res.stdout + res.stderr)
                raise RuntimeError(f"nvcc failed for {src}")
            if verbose:
                sys.stdout.write(res.stderr)
            relink = True
    if relink:
        cmd = [nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", LIB, *objs, "-lcudart_static", "-lrt",
               "-lpthread", "-ldl"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            sys.stderr.write(res.stdout + res.stderr)
            raise RuntimeError("link of libuttt_b200.so failed")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.verbose))
