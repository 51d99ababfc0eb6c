"""Host-side engine checks that need no GPU: the library loads and exports its
ABI, the fusion pass and the arena planner behave like the reference's, and
the per-model library validates calls with the reference's status codes."""

import ctypes
import json
import os
import re
import subprocess

import numpy as np
import pytest
import torch
import torch.nn as nn

from forgetune_b200 import InvalidShapeError, _native, compile_model, workloads
from forgetune_b200.build_native import LIB_PATH
from forgetune_b200.frontend import export_to_ir
from forgetune_b200.graph_blob import serialize

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "forgetune_b200.h")
GOLDEN = json.load(open(os.path.join(REPO, "tests", "golden", "golden.json")))


def header_symbols(prefix):
    src = open(HEADER).read()
    return sorted(set(re.findall(r"FORGETUNE_EXPORT\s+[\w\s\*]+?\b(%s\w*)\s*\(" % prefix, src)))


def exported(path):
    out = subprocess.run(["nm", "-D", "--defined-only", path], capture_output=True, text=True, check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if line.strip()}


def test_engine_library_exports_every_declared_symbol():
    syms = header_symbols("ftb_")
    assert len(syms) >= 20
    have = exported(LIB_PATH)
    missing = [s for s in syms if s not in have]
    assert not missing, missing
    _native.lib()  # loads and binds every signature


def blob_of(model, x, dynamic=True, max_batch=128, fusion=True, variant_bias_first=True, fold=True):
    ir = export_to_ir(model, (x,), dynamic_batch=dynamic, max_batch_size=max_batch)
    return serialize(ir, enable_fusion=fusion, bias_first_fused=variant_bias_first, fold_epilogues=fold)


@pytest.fixture(scope="module")
def tiny_compiled(tmp_path_factory):
    m = workloads.tiny_mlp()
    cm = compile_model(m, (workloads.seeded_input((4, 784)),), output_dir=str(tmp_path_factory.mktemp("tiny")),
                       autotune=False, kernel_variant="fused_ikj", enable_fusion=True, dynamic_batch=True,
                       max_batch_size=128, verify=False)
    yield cm
    cm.close()


def test_model_library_exports_reference_abi(tiny_compiled):
    have = exported(tiny_compiled.manifest()["artifacts"]["shared_library"])
    want = header_symbols("forgetune_") + ["forgetune_run"]
    missing = [s for s in want if s not in have]
    assert not missing, missing
    # nothing but the ABI is exported
    assert all(s.startswith("forgetune_") for s in have), sorted(s for s in have if not s.startswith("forgetune_"))


def test_status_codes_without_gpu(tiny_compiled):
    """Validation precedes any device work (src/codegen.cpp:729-741, 1001-1008)."""
    rt = tiny_compiled._runtime
    x = np.ones((2, 784), np.float32)
    y = np.zeros((2, 10), np.float32)
    xp, yp = x.ctypes.data, y.ctypes.data
    assert rt.run_v2_fn(xp, x.size, yp, y.size, 0) == -2          # B <= 0 first
    assert rt.run_v2_fn(None, x.size, None, y.size, 0) == -2
    assert rt.run_v2_fn(None, x.size, yp, y.size, 2) == -1
    assert rt.run_v2_fn(xp, x.size, None, y.size, 2) == -1
    assert rt.run_v2_fn(xp, x.size - 1, yp, y.size, 2) == -2
    assert rt.run_v2_fn(xp, x.size, yp, y.size - 1, 2) == -3
    assert rt.run_v2_fn(xp, 784 * 129, yp, 10 * 129, 129) == -2   # B > max_batch
    assert rt.run_v1_fn(xp, 783, yp, y.size) == -2                 # not a multiple of the sample size
    assert rt.run_v1_fn(xp, 0, yp, 0) == -2
    assert rt.lib.forgetune_is_dynamic() == 1
    assert rt.lib.forgetune_max_batch() == 128
    # python-side checks of the NativeRuntime mirror
    with pytest.raises(TypeError):
        tiny_compiled.run(np.ones((2, 784), np.float64))
    with pytest.raises(InvalidShapeError):
        tiny_compiled.run(np.ones((0, 784), np.float32))
    with pytest.raises(InvalidShapeError):
        tiny_compiled.run(np.ones((129, 784), np.float32))
    with pytest.raises(InvalidShapeError):
        tiny_compiled.run(np.ones((4, 783), np.float32))


def test_static_model_status_codes(tmp_path):
    torch.manual_seed(42)
    m = nn.Sequential(nn.Linear(8, 4), nn.ReLU()).eval()
    cm = compile_model(m, (torch.randn(2, 8),), output_dir=str(tmp_path), autotune=False, dynamic_batch=False,
                       verify=False)
    rt = cm._runtime
    assert rt.lib.forgetune_is_dynamic() == 0 and rt.lib.forgetune_max_batch() == 2
    x = np.ones((2, 8), np.float32)
    y = np.zeros((2, 4), np.float32)
    assert rt.run_v2_fn(x.ctypes.data, 16, y.ctypes.data, 8, 3) == -2   # B must equal the static batch
    assert rt.run_v1_fn(x.ctypes.data, 15, y.ctypes.data, 8) == -2
    assert rt.run_v1_fn(x.ctypes.data, 16, y.ctypes.data, 7) == -3
    assert rt.run_v1_fn(None, 16, y.ctypes.data, 8) == -1
    cm.close()


def test_bad_blobs_are_rejected():
    blob = bytearray(blob_of(nn.Sequential(nn.Linear(8, 4)).eval(), torch.randn(2, 8)))
    assert _native.describe_blob(bytes(blob))["steps"]
    bad = bytearray(blob)
    bad[0:8] = b"NOTGRAPH"
    with pytest.raises(Exception):
        _native.describe_blob(bytes(bad))
    with pytest.raises(Exception):
        _native.describe_blob(bytes(blob[:50]))


def ops_of(desc):
    return [(n["op"], n["epi"]) for n in desc["nodes"] if n["op"] not in ("INPUT", "CONST")]


EPI_BIAS_FIRST, EPI_BIAS_LAST, EPI_RELU_PRE, EPI_RESIDUAL, EPI_RELU_POST = 1, 2, 4, 8, 16


def test_fusion_tiny_mlp():
    d = _native.describe_blob(blob_of(workloads.tiny_mlp(), torch.randn(2, 784)))
    assert ops_of(d) == [("GEMM", EPI_BIAS_FIRST | EPI_RELU_PRE), ("GEMM", EPI_BIAS_FIRST | EPI_RELU_PRE),
                         ("GEMM", EPI_BIAS_LAST)]
    # naive_ijk order: the fused layers add the bias after the sum
    d = _native.describe_blob(blob_of(workloads.tiny_mlp(), torch.randn(2, 784), variant_bias_first=False))
    assert ops_of(d)[0] == ("GEMM", EPI_BIAS_LAST | EPI_RELU_PRE)


def test_fusion_residual_epilogue():
    d = _native.describe_blob(blob_of(workloads.residual_mlp(), torch.randn(2, 512)))
    ops = ops_of(d)
    assert len(ops) == 10  # stem, 4 x (fc1, fc2 + residual), head: one launch each
    assert ops[2] == ("GEMM", EPI_BIAS_LAST | EPI_RESIDUAL)
    assert all(k == "GEMM" for k, _ in ops)


def test_fusion_cnn_flatten_is_a_view():
    d = _native.describe_blob(blob_of(workloads.small_cnn(), torch.randn(2, 3, 32, 32)))
    ops = ops_of(d)
    assert [k for k, _ in ops] == ["CONV", "CONV", "CONV", "FLATTEN", "GEMM", "GEMM"]
    flat = [n for n in d["nodes"] if n["op"] == "FLATTEN"][0]
    assert flat["alias_of"] >= 0
    assert len(d["steps"]) == 5  # the view launches nothing


def test_unfused_graph_keeps_separate_nodes():
    d = _native.describe_blob(blob_of(workloads.tiny_mlp(), torch.randn(2, 784), fusion=False,
                                      variant_bias_first=False))
    assert [k for k, _ in ops_of(d)] == ["GEMM", "ADD", "RELU", "GEMM", "ADD", "RELU", "GEMM", "ADD"]


@pytest.mark.parametrize("name,sample,max_batch", [("tiny_mlp", (784,), 65536), ("residual_mlp", (512,), 1024),
                                                   ("small_cnn", (3, 32, 32), 256)])
def test_arena_plan_equals_reference_planner(name, sample, max_batch):
    """With only the reference's fusion, the interval colouring reproduces the
    reference planner's arena size and offsets (src/memory_planner.cpp:106-174)."""
    model = workloads.WORKLOADS[name][0]()
    d = _native.describe_blob(blob_of(model, torch.randn((2,) + sample), max_batch=max_batch, fold=False))
    ref = GOLDEN["reference_plans"][name]
    assert d["arena_bytes"] == ref["arena_bytes"]
    assert [a["offset"] for a in d["allocs"]] == ref["offsets_bytes"]
    # with epilogue folding the arena can only shrink
    d2 = _native.describe_blob(blob_of(model, torch.randn((2,) + sample), max_batch=max_batch))
    assert d2["arena_bytes"] <= d["arena_bytes"]


def test_workspace_budget_enforced(tmp_path):
    with pytest.raises(ValueError, match="workspace"):
        compile_model(workloads.tiny_mlp(), (torch.randn(2, 784),), output_dir=str(tmp_path), autotune=False,
                      dynamic_batch=True, max_batch_size=1_000_000, verify=False)


def test_compile_model_argument_checks(tmp_path):
    m = workloads.tiny_mlp()
    x = torch.randn(2, 784)
    with pytest.raises(ValueError):
        compile_model(m, (x,), output_dir=str(tmp_path), autotune=False, max_batch_size=0)
    with pytest.raises(ValueError):
        compile_model(m, (x,), output_dir=str(tmp_path), autotune=False, kernel_variant="fused_ikj",
                      enable_fusion=False)
    with pytest.raises(ValueError):
        compile_model(m, (x,), output_dir=str(tmp_path), autotune=True, kernel_variant="naive_ijk")
    with pytest.raises(ValueError):
        compile_model(m, (x,), output_dir=str(tmp_path), autotune=False, gpu_kernel="triton")


def _reference_python():
    from oracle.build_ref import reference_root
    return os.path.join(reference_root(), "python")


REFERENCE_PY = _reference_python()


@pytest.mark.skipif(not os.path.isdir(REFERENCE_PY), reason="reference checkout not present")
def test_reference_native_runtime_binds_artifact(tiny_compiled):
    """The reference's own ctypes loader (python/forgetune/runtime.py) binds a
    compiled artifact unchanged: same symbols, same contract checks."""
    import importlib
    import sys
    sys.path.insert(0, REFERENCE_PY)
    try:
        ref_runtime = importlib.import_module("forgetune.runtime")
        ref_errors = importlib.import_module("forgetune.errors")
    finally:
        sys.path.remove(REFERENCE_PY)
    so = tiny_compiled.manifest()["artifacts"]["shared_library"]
    rt = ref_runtime.NativeRuntime(so, (-1, 784), (-1, 10))
    assert rt.is_dynamic and rt.max_batch_size == 128
    with pytest.raises(ref_errors.InvalidShapeError):
        rt.run(np.ones((129, 784), np.float32))
    with pytest.raises(TypeError):
        rt.run(np.ones((2, 784), np.float64))
    x = np.ones((2, 784), np.float32)
    if _native.device_count() == 0:
        with pytest.raises(ref_errors.ForgeTuneRuntimeError, match="-5"):
            rt.run(x)
    else:
        np.testing.assert_array_equal(rt.run(x), tiny_compiled.run(x))


def _mlp_marks(model, x):
    steps = _native.describe_blob(blob_of(model, x))["steps"]
    return [(s["mlp_step"], s["mlp_of"], s["head_step"], s["head_of"]) for s in steps]


def test_two_layer_candidates():
    """Step pairs one launch may compute together (first layer 129..256 wide
    feeding only the second, 64..128 wide, column biases / ReLUs), and the
    second layer's small head; everything else stays separate launches."""
    # the tiny MLP: layers 0 and 1 together, the head (step 2) in layer 1's epilogue
    assert _mlp_marks(workloads.tiny_mlp(), torch.randn(2, 784)) == [(1, -1, -1, -1), (-1, 0, 2, -1),
                                                                      (-1, -1, -1, 1)]
    # second layer too narrow for the pair (it is a head of the first instead)
    m = nn.Sequential(nn.Linear(64, 256), nn.ReLU(), nn.Linear(256, 10)).eval()
    assert _mlp_marks(m, torch.randn(2, 64)) == [(-1, -1, 1, -1), (-1, -1, -1, 0)]
    # first layer too wide for layer 1's TMEM columns, or too narrow to be worth it
    for n1 in (512, 128):
        m = nn.Sequential(nn.Linear(64, n1), nn.ReLU(), nn.Linear(n1, 128), nn.ReLU()).eval()
        assert all(t[0] == -1 and t[1] == -1 for t in _mlp_marks(m, torch.randn(2, 64))), n1
    # three wide layers: only the first pair (a step is in at most one pair)
    m = nn.Sequential(nn.Linear(64, 200), nn.ReLU(), nn.Linear(200, 100), nn.ReLU(), nn.Linear(100, 256),
                      nn.ReLU(), nn.Linear(256, 64)).eval()
    marks = _mlp_marks(m, torch.randn(2, 64))
    assert marks[0][0] == 1 and marks[1][1] == 0 and marks[2][0] == 3 and marks[3][1] == 2
    # a layer with a residual epilogue (and the layer whose output it also
    # reads) stays a separate launch
    class Res(nn.Module):
        def __init__(self):
            super().__init__()
            self.fc = nn.Linear(256, 256)

        def forward(self, x):
            return torch.relu(self.fc(x)) + x

    m = nn.Sequential(nn.Linear(64, 256), nn.ReLU(), Res(), nn.Linear(256, 128), nn.ReLU()).eval()
    assert all(t[0] == -1 and t[1] == -1 for t in _mlp_marks(m, torch.randn(2, 64)))
