"""Build libforgetune_b200.so in-tree with nvcc for sm_100a.

    python -m forgetune_b200.build_native [--force]

The library holds the engine (graph blob, fusion, arena planner), every CUDA
kernel and the C ABI declared in include/forgetune_b200.h.  It is written to
forgetune_b200/lib/ and linked (with an rpath) by every per-model shim.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(REPO, "include")
LIB_DIR = os.path.join(PKG, "lib")
LIB_PATH = os.path.join(LIB_DIR, "libforgetune_b200.so")

SOURCES = ["runtime.cu", "engine.cpp"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.isfile(cand):
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put CUDA on PATH)")


def _inputs():
    files = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cuh", ".cpp", ".hpp", ".h"))]
    files.append(os.path.join(INCLUDE, "forgetune_b200.h"))
    return files


def up_to_date() -> bool:
    if not os.path.isfile(LIB_PATH):
        return False
    t = os.path.getmtime(LIB_PATH)
    return all(os.path.getmtime(f) <= t for f in _inputs())


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB_PATH
    os.makedirs(LIB_DIR, exist_ok=True)
    tmp = LIB_PATH + ".tmp%d" % os.getpid()
    cmd = [nvcc(), "-std=c++17", "-O3", "-lineinfo"] + ARCH_FLAGS + [
        "-I", INCLUDE, "-Xcompiler", "-fPIC,-fvisibility=hidden", "-shared",
        "-o", tmp] + [os.path.join(CSRC, s) for s in SOURCES]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed (%d):\n%s\n%s" % (r.returncode, r.stdout[-4000:], r.stderr[-8000:]))
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=True))
    return 0


if __name__ == "__main__":
    sys.exit(main())
