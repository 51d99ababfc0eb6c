#!/usr/bin/env python3
"""Generate the golden vectors in this directory from the reference runtime.

Runs the reference's own generated CPU runtime (oracle/_ref/<workload>_<variant>.so,
built by oracle/build_ref.py from the reference sources) through its C ABI
``forgetune_run_v2`` on the seeded inputs of forgetune_b200.workloads and stores:

  golden.npz   full outputs for the small cases, sampled rows for the
               B=65536 tiny-MLP sweep point, and the edge-case outputs;
  golden.json  SHA-256 of every input, of the weights and of every full output,
               so a torch RNG drift or an output mismatch is detected even where
               only sampled rows are stored.

Inputs are not stored: they are regenerated from their seeds and checked
against the stored SHA-256.  Run in a checkout that has oracle/_ref built:
    python tests/golden/make_golden.py
"""

from __future__ import annotations

import ctypes
import hashlib
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from forgetune_b200 import workloads  # noqa: E402

REF_DIR = os.path.join(REPO, "oracle", "_ref")
VARIANTS = ("fused_ikj", "naive_ijk")

# (workload, B, input kind) -- kinds: seeded N(0,1), zeros, const -100, seeded x 1e3
CASES = [
    ("tiny_mlp", 1, "seeded"),
    ("tiny_mlp", 7, "seeded"),
    ("tiny_mlp", 8, "seeded"),
    ("tiny_mlp", 64, "seeded"),
    ("tiny_mlp", 128, "seeded"),
    ("tiny_mlp", 4096, "seeded"),
    ("tiny_mlp", 65536, "seeded"),
    ("tiny_mlp", 5, "zeros"),
    ("tiny_mlp", 3, "neg100"),
    ("tiny_mlp", 16, "wide_range"),
    ("tiny_mlp", 64, "wide_range"),
    ("tiny_mlp", 4096, "wide_range"),
    ("residual_mlp", 1024, "seeded"),
    ("residual_mlp", 3, "wide_range"),
    ("residual_mlp", 1024, "wide_range"),
    ("small_cnn", 1, "seeded"),
    ("small_cnn", 256, "seeded"),
    ("small_cnn", 2, "neg100"),
    ("small_cnn", 256, "wide_range"),
    ("op_mix", 1, "seeded"),
    ("op_mix", 64, "seeded"),
    ("op_mix", 300, "seeded"),
    ("op_mix", 64, "wide_range"),
]
# input scale of each kind: the wide-range inputs are the seeded draw x 1e3
INPUT_SCALE = {"seeded": 1.0, "zeros": 1.0, "neg100": 1.0, "wide_range": 1e3}
FULL_OUTPUT_LIMIT = 4096  # store every row up to this batch, sampled rows beyond
SAMPLED_ROWS = 256


def make_input(name: str, B: int, kind: str) -> np.ndarray:
    shape = (B,) + tuple(workloads.WORKLOADS[name][1])
    if kind == "seeded":
        return workloads.seeded_input(shape).numpy()
    if kind == "zeros":
        return np.zeros(shape, np.float32)
    if kind == "neg100":
        return np.full(shape, -100.0, np.float32)
    if kind == "wide_range":
        return (workloads.seeded_input(shape).numpy() * np.float32(1e3)).astype(np.float32)
    raise ValueError(kind)


def sampled_rows(B: int) -> np.ndarray:
    """Deterministic sample: first, last and evenly spaced rows."""
    return np.unique(np.linspace(0, B - 1, SAMPLED_ROWS).astype(np.int64))


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def weights_sha(model) -> str:
    h = hashlib.sha256()
    for k, v in model.state_dict().items():
        h.update(k.encode())
        h.update(v.detach().numpy().astype(np.float32).tobytes())
    return h.hexdigest()


def ref_run(so_path: str, x: np.ndarray, out_feats: int) -> np.ndarray:
    lib = ctypes.CDLL(so_path)
    fn = lib.forgetune_run_v2
    fn.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int64]
    fn.restype = ctypes.c_int
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty((x.shape[0], out_feats), np.float32)
    rc = fn(x.ctypes.data, x.size, y.ctypes.data, y.size, x.shape[0])
    if rc != 0:
        raise RuntimeError("reference runtime returned %d" % rc)
    return y


def reference_plan(name: str) -> dict:
    """Arena size and buffer offsets the reference planner chose, read from the
    kernel.cpp its code generator emitted (``acquire(<bytes>)`` and
    ``buf_<id> = arena + <float offset>`` lines, in execution order)."""
    import re
    path = os.path.join(REF_DIR, "_src", name, "kernel_fused_ikj.cpp")
    with open(path) as f:
        src = f.read()
    arena = int(re.search(r"g_thread_arena_pool\.acquire\((\d+)\)", src).group(1))
    offs = [int(m.group(2)) * 4 for m in re.finditer(r"float\* buf_(\d+) = arena \+ (\d+);", src)]
    return {"arena_bytes": arena, "offsets_bytes": offs}


def main() -> int:
    arrays = {}
    meta = {"torch": torch.__version__, "weights_sha256": {}, "cases": [], "reference_plans": {}}
    for name in ("tiny_mlp", "residual_mlp", "small_cnn", "op_mix"):
        meta["reference_plans"][name] = reference_plan(name)
    models = {}
    for name, B, kind in CASES:
        if name not in models:
            models[name] = workloads.WORKLOADS[name][0]()
            meta["weights_sha256"][name] = weights_sha(models[name])
        x = make_input(name, B, kind)
        key = "%s_B%d_%s" % (name, B, kind)
        case = {"key": key, "workload": name, "batch": B, "input": kind, "input_scale": INPUT_SCALE[kind],
                "input_sha256": sha(x), "outputs": {}}
        rows = None if B <= FULL_OUTPUT_LIMIT else sampled_rows(B)
        if rows is not None:
            arrays[key + "__rows"] = rows
        for v in VARIANTS:
            y = ref_run(os.path.join(REF_DIR, "%s_%s.so" % (name, v)), x, 10)
            case["outputs"][v] = {"sha256": sha(y), "shape": list(y.shape)}
            arrays[key + "__" + v] = y if rows is None else y[rows]
        meta["cases"].append(case)
        print("golden", key, flush=True)
    np.savez_compressed(os.path.join(HERE, "golden.npz"), **arrays)
    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump(meta, f, indent=1)
    return 0


if __name__ == "__main__":
    sys.exit(main())
