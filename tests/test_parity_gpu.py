"""GPU parity: the CUDA forward pass against the reference runtime's golden
vectors and the CPU oracle, through the C ABI of the compiled model.

* ``simt_exact``: separately rounded mul/add in the reference's order --
  every golden output must match bit for bit (SHA-256 of the full output,
  B=65536 included).
  The op-mix workload's SIGMOID / TANH use CUDA's expf / tanhf where the
  reference uses the C library's, which may differ in the last bit: that
  workload is held to the tolerance below under every policy.
* default (``auto``), ``simt`` and ``tcgen05``, on every golden case:
  np.allclose(atol=1e-4 * s, rtol=1e-4), the reference's own tolerance
  (python/forgetune/compiler.py:230-231) with atol scaled by the input's scale
  s (1 for N(0,1) inputs, 1e3 for the wide-range inputs).  At x 1e3 the fixed
  atol is below fp32's own rounding noise: the reference's two variants fail
  it against each other (tests/test_oracle_golden.py), so no other operation
  order can meet it; the wide-range cases at 17 rows and more run on the
  tensor cores under ``auto``.
* run-to-run and batch-size invariance: bitwise.
"""

import hashlib
import json
import os

import numpy as np
import pytest
import torch

from forgetune_b200 import _native, compile_model, workloads
from oracle import oracle
from tests.golden.make_golden import make_input, sha

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
META = json.load(open(os.path.join(HERE, "golden", "golden.json")))
GOLD = np.load(os.path.join(HERE, "golden", "golden.npz"))
ATOL = RTOL = 1e-4
MAX_BATCH = {"tiny_mlp": 65536, "residual_mlp": 1024, "small_cnn": 256, "op_mix": 512}
TRANSCENDENTAL = {"op_mix"}  # SIGMOID / TANH: libm and CUDA may differ by an ulp
_MODELS = {}
_COMPILED = {}


def model(name):
    if name not in _MODELS:
        _MODELS[name] = workloads.WORKLOADS[name][0]()
    return _MODELS[name]


def compiled(name, variant, policy, tmp_root):
    key = (name, variant, policy)
    if key not in _COMPILED:
        shape = workloads.WORKLOADS[name][1]
        _COMPILED[key] = compile_model(
            model(name), (workloads.seeded_input((2,) + tuple(shape)),),
            output_dir=os.path.join(tmp_root, "%s_%s_%s" % key), autotune=False, kernel_variant=variant,
            enable_fusion=True, dynamic_batch=True, max_batch_size=MAX_BATCH[name],
            max_workspace_bytes=4 << 30, gpu_kernel=policy)
    return _COMPILED[key]


@pytest.fixture(scope="module")
def tmp_root(tmp_path_factory):
    d = str(tmp_path_factory.mktemp("parity"))
    yield d
    for cm in _COMPILED.values():
        cm.close()
    _COMPILED.clear()


CASES = [(c["key"], v) for c in META["cases"] for v in c["outputs"]]


@pytest.mark.parametrize("key,variant", CASES)
def test_exact_policy_bitwise_equals_reference(key, variant, tmp_root):
    case = next(c for c in META["cases"] if c["key"] == key)
    cm = compiled(case["workload"], variant, "simt_exact", tmp_root)
    x = make_input(case["workload"], case["batch"], case["input"])
    assert sha(x) == case["input_sha256"]
    y = cm.run(x)
    if case["workload"] in TRANSCENDENTAL:
        rows = GOLD[key + "__rows"] if (key + "__rows") in GOLD.files else None
        want = GOLD[key + "__" + variant]
        got = y if rows is None else y[rows]
        atol = ATOL * case.get("input_scale", 1.0)
        assert np.allclose(got, want, atol=atol, rtol=RTOL), float(np.max(np.abs(got - want)))
        return
    assert sha(y) == case["outputs"][variant]["sha256"], "output differs from the reference runtime"


FAST_CASES = [(c["key"], p) for c in META["cases"] for p in ("auto", "simt", "tcgen05")]


@pytest.mark.parametrize("key,policy", FAST_CASES)
def test_fast_policies_within_reference_tolerance(key, policy, tmp_root):
    case = next(c for c in META["cases"] if c["key"] == key)
    cm = compiled(case["workload"], "fused_ikj", policy, tmp_root)
    x = make_input(case["workload"], case["batch"], case["input"])
    y = cm.run(x)
    rows = GOLD.get(key + "__rows") if (key + "__rows") in GOLD.files else None
    want = GOLD[key + "__fused_ikj"]
    got = y if rows is None else y[rows]
    atol = ATOL * case.get("input_scale", 1.0)
    err = np.abs(got.astype(np.float64) - want) - (atol + RTOL * np.abs(want.astype(np.float64)))
    assert np.allclose(got, want, atol=atol, rtol=RTOL), (
        "max |err| %.3g, worst excess over the band %.3g" % (float(np.max(np.abs(got - want))), float(err.max())))


@pytest.mark.parametrize("policy", ["auto", "simt", "simt_exact", "tcgen05"])
def test_run_to_run_and_batch_invariance(policy, tmp_root):
    cm = compiled("tiny_mlp", "fused_ikj", policy, tmp_root)
    x = make_input("tiny_mlp", 65536, "seeded")
    a = cm.run(x)
    b = cm.run(x)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    # Rows are independent in every kernel, so the same rows inside a batch
    # that selects the same kernels give the same bits.  "simt_exact" uses one
    # kernel family for every size; "simt" uses the split-K kernel up to 16
    # rows and register tiles (narrow-N kernel for the head) above; "auto"
    # adds the tensor cores from 17 rows and split-K for few, long-K tiles.
    slices = {"simt_exact": ((0, 1), (100, 357), (4096, 8192), (65000, 65536)),
              "simt": ((100, 357), (4096, 8192), (65000, 65536)),
              "auto": (), "tcgen05": ()}[policy]
    for lo, hi in slices:
        part = cm.run(np.ascontiguousarray(x[lo:hi]))
        assert np.array_equal(part.view(np.uint32), a[lo:hi].view(np.uint32)), (lo, hi)


def test_unfused_graph_matches_oracle(tmp_path):
    m = model("tiny_mlp")
    cm = compile_model(m, (workloads.seeded_input((2, 784)),), output_dir=str(tmp_path), autotune=False,
                       kernel_variant="naive_ijk", enable_fusion=False, dynamic_batch=True, max_batch_size=256,
                       gpu_kernel="simt_exact")
    x = make_input("tiny_mlp", 77, "seeded")
    want = oracle.run_model(m, x, "naive_ijk", fusion=False)
    assert np.array_equal(cm.run(x).view(np.uint32), want.view(np.uint32))
    cm.close()


def test_device_resident_entry_point(tmp_root):
    cm = compiled("small_cnn", "fused_ikj", "auto", tmp_root)
    x = make_input("small_cnn", 256, "seeded")
    xd = torch.from_numpy(x).cuda()
    yd = cm.run_device(xd)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(yd.cpu().numpy(), cm.run(x))


def test_philox_device_matches_host():
    n = 1 << 16
    d = torch.empty(n + 13, dtype=torch.float32, device="cuda")
    _native.philox_normal(d.data_ptr(), 1, 12345, n + 13)
    torch.cuda.synchronize()
    host = oracle.philox_normal(1, 12345, n + 13)
    np.testing.assert_allclose(d.cpu().numpy(), host, atol=2e-6, rtol=2e-6)
    # split generation equals one-shot generation, bitwise
    e = torch.empty(n + 13, dtype=torch.float32, device="cuda")
    _native.philox_normal(e.data_ptr(), 1, 12345, 1001)
    _native.philox_normal(e.data_ptr() + 1001 * 4, 1, 12345 + 1001, n + 13 - 1001)
    torch.cuda.synchronize()
    assert torch.equal(d, e)


def test_wide_mlp_full_batch_sampled_rows(tmp_path):
    """Wide MLP at box scale on one GPU: B=262144 generated on the device,
    64 sampled rows checked against the oracle (the reference interpreter's
    bias-last order, src/interpreter.cpp:8-66)."""
    m = workloads.wide_mlp()
    B = 262144
    cm = compile_model(m, (workloads.seeded_input((2, 4096)),), output_dir=str(tmp_path), autotune=False,
                       enable_fusion=True, dynamic_batch=True, max_batch_size=B, max_workspace_bytes=64 << 30,
                       gpu_kernel="auto", verify=False)
    with open(cm.manifest()["artifacts"]["graph_blob"], "rb") as f:
        eng = _native.EngineModel(f.read())
    x = torch.empty(B * 4096, dtype=torch.float32, device="cuda")
    y = torch.empty(B * 4096, dtype=torch.float32, device="cuda")
    _native.philox_normal(x.data_ptr(), 1, 0, B * 4096)
    eng.run_device(x.data_ptr(), B * 4096, y.data_ptr(), B * 4096, B)
    torch.cuda.synchronize()
    rows = np.unique(np.linspace(0, B - 1, 64).astype(np.int64))
    xr = x.view(B, 4096)[torch.from_numpy(rows).cuda()].cpu().numpy()
    got = y.view(B, 4096)[torch.from_numpy(rows).cuda()].cpu().numpy()
    want = oracle.run_model(m, xr, "naive_ijk")
    assert np.allclose(got, want, atol=ATOL, rtol=RTOL), float(np.max(np.abs(got - want)))
    assert np.isfinite(y.view(B, 4096)[-1].cpu().numpy()).all()
    eng.close()
    cm.close()
