#!/usr/bin/env python3
"""Build the reference's own CPU runtime for the measured workloads -- TEST INFRASTRUCTURE ONLY.

Recipe (reads the read-only reference checkout, writes only into oracle/_ref/):
  1. g++ the reference engine CLI from its own sources
     (src/{ir,graph_verifier,pass_manager,optimizer,fusion,memory_planner,
     json_io,codegen,interpreter,main}.cpp) -> oracle/_ref/forgetune_engine.
  2. For each workload, export it with the reference's Python frontend
     (python/forgetune/export_frontend.py:47, dynamic batch), write graph.json,
     run `forgetune_engine --compile ... --variant V --fusion` (src/main.cpp:88-183)
     and compile the emitted kernel.cpp with the reference's own flags
     (python/forgetune/native_compiler.py:163-177:
     -shared -fPIC -std=c++17 -O2 -Wall -Wextra -fno-signed-zeros)
     -> oracle/_ref/<workload>_<variant>.so.
The .so files export the reference C ABI (include/forgetune/forgetune_abi.h)
and are the reference runtime used as the CPU baseline and to pin the oracle.
They are git-ignored but travel with the working tree; the intermediate
graph.json / kernel.cpp files stay in oracle/_ref/_src/, which does not travel.

Usage: python oracle/build_ref.py [--reference DIR] [--only tiny_mlp]

The reference checkout is DIR, else $FORGETUNE_REFERENCE, else /root/reference
(reference_root() below is the one place the default is named).
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
OUT = os.path.join(HERE, "_ref")

ENGINE_SOURCES = ["ir", "graph_verifier", "pass_manager", "optimizer", "fusion",
                  "memory_planner", "json_io", "codegen", "interpreter", "main"]

# workload -> max_batch_size compiled into the reference .so
TARGETS = {
    "tiny_mlp": 65536,
    "residual_mlp": 1024,
    "small_cnn": 256,
    "op_mix": 512,
}
VARIANTS = ("fused_ikj", "naive_ijk")


def reference_root() -> str:
    """The reference checkout: $FORGETUNE_REFERENCE, else the default mount."""
    return os.environ.get("FORGETUNE_REFERENCE", "/root/reference")


def build_engine(ref: str) -> str:
    exe = os.path.join(OUT, "forgetune_engine")
    srcs = [os.path.join(ref, "src", s + ".cpp") for s in ENGINE_SOURCES]
    if os.path.isfile(exe) and all(os.path.getmtime(exe) >= os.path.getmtime(s) for s in srcs):
        return exe
    cmd = ["g++", "-O2", "-std=c++17", "-I", os.path.join(ref, "include")] + srcs + ["-o", exe]
    print("[build_ref]", " ".join(cmd[:6]), "...", flush=True)
    subprocess.check_call(cmd)
    return exe


def export_graph(ref: str, name: str, max_batch: int, path: str) -> None:
    sys.path.insert(0, os.path.join(ref, "python"))
    sys.path.insert(0, REPO)
    from forgetune.export_frontend import export_to_forgetune_ir  # reference frontend
    from forgetune_b200 import workloads

    builder, sample_shape, _ = workloads.WORKLOADS[name]
    model = builder()
    x = workloads.seeded_input((2,) + tuple(sample_shape))
    g = export_to_forgetune_ir(model, (x,), dynamic_batch=True, max_batch_size=max_batch)
    with open(path, "w") as f:
        f.write(g.to_json())


def build_one(ref: str, engine: str, name: str, max_batch: int) -> None:
    gdir = os.path.join(OUT, "_src", name)
    os.makedirs(gdir, exist_ok=True)
    gjson = os.path.join(gdir, "graph.json")
    if not os.path.isfile(gjson):
        t = time.time()
        export_graph(ref, name, max_batch, gjson + ".tmp")
        os.replace(gjson + ".tmp", gjson)
        print("[build_ref] exported %s in %.1fs" % (name, time.time() - t), flush=True)
    for variant in VARIANTS:
        so = os.path.join(OUT, "%s_%s.so" % (name, variant))
        if os.path.isfile(so):
            continue
        cpp = os.path.join(gdir, "kernel_%s.cpp" % variant)
        subprocess.check_call([engine, "--compile", gjson, "-o", cpp, "--variant", variant,
                               "--fusion", "--max-batch-size", str(max_batch),
                               "--max-workspace-bytes", str(16 << 30)],
                              stdout=subprocess.DEVNULL)
        t = time.time()
        subprocess.check_call(["g++", "-shared", "-fPIC", "-o", so + ".tmp", cpp, "-std=c++17",
                               "-O2", "-Wall", "-Wextra", "-fno-signed-zeros"])
        os.replace(so + ".tmp", so)
        print("[build_ref] compiled %s in %.1fs" % (os.path.basename(so), time.time() - t), flush=True)


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None)
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    args.reference = args.reference or reference_root()
    if not os.path.isdir(os.path.join(args.reference, "src")):
        print("[build_ref] reference checkout not found at %s; nothing to build" % args.reference)
        return 0
    os.makedirs(OUT, exist_ok=True)
    engine = build_engine(args.reference)
    mpath = os.path.join(OUT, "manifest.json")
    meta = {}
    if os.path.isfile(mpath):
        with open(mpath) as f:
            meta = json.load(f)
    for name, mb in TARGETS.items():
        if args.only and name != args.only:
            continue
        build_one(args.reference, engine, name, mb)
        meta[name] = {"max_batch": mb, "variants": list(VARIANTS)}
    with open(mpath, "w") as f:
        json.dump(meta, f, indent=1)
    return 0


if __name__ == "__main__":
    sys.exit(main())
