"""The small-batch chain kernel: the whole forward pass of a chain of dense
layers in one launch for at most 16 rows (csrc/chain_gemv.cuh), with every
warp's weight rows cached in shared memory when they fit and streamed from
L2 otherwise.

* it is the kernel that runs (one kernel per forward) for the tiny and the
  residual MLP at 1..16 rows, and the outputs match the oracle (the
  reference's arithmetic) within the reference tolerance;
* results are bitwise identical run to run;
* launch lists it cannot run (K not a multiple of 4, an elementwise node,
  an input pointer that is not 16-byte aligned) keep the per-layer kernels;
* a wait for another CTA's values that runs out (up to 8 rows each value a
  tagged word and the layers hand over without grid barriers; at 16 rows a
  grid barrier) is reported as -5 and the context then computes correctly
  again (no GPU fault).
"""

import numpy as np
import pytest
import torch
import torch.nn as nn

from forgetune_b200 import _native, compile_model, workloads
from oracle import oracle

pytestmark = pytest.mark.gpu

ATOL = RTOL = 1e-4


def engine(model, sample_shape, tmp_path, max_batch=64, policy="auto"):
    cm = compile_model(model, (torch.randn((2,) + tuple(sample_shape)),), output_dir=str(tmp_path), autotune=False,
                       enable_fusion=True, kernel_variant="fused_ikj", dynamic_batch=True, max_batch_size=max_batch,
                       gpu_kernel=policy, verify=False)
    with open(cm.manifest()["artifacts"]["graph_blob"], "rb") as f:
        eng = _native.EngineModel(f.read())
    eng.set_devices([torch.cuda.current_device()])
    return cm, eng


def run_dev(eng, x_np, out_f):
    B = x_np.shape[0]
    x = torch.from_numpy(np.ascontiguousarray(x_np)).cuda().reshape(-1)
    y = torch.full((B * out_f,), float("nan"), dtype=torch.float32, device="cuda")
    eng.run_device(x.data_ptr(), x.numel(), y.data_ptr(), y.numel(), B, 0)
    torch.cuda.synchronize()
    return y.cpu().numpy().reshape(B, out_f)


@pytest.mark.parametrize("name", ["tiny_mlp", "residual_mlp"])
@pytest.mark.parametrize("policy", ["auto", "simt"])
def test_chain_runs_and_matches_oracle(name, policy, tmp_path):
    builder, shape, _ = workloads.WORKLOADS[name]
    m = builder()
    cm, eng = engine(m, shape, tmp_path, policy=policy)
    x_all = workloads.seeded_input((16,) + tuple(shape)).numpy()
    for B in (1, 2, 7, 16):
        got = run_dev(eng, x_all[:B], 10)
        assert eng.graph_kernels() == 1, "the chain kernel should be the forward's only kernel"
        want = oracle.run_model(m, x_all[:B], "fused_ikj")
        assert np.allclose(got, want, atol=ATOL, rtol=RTOL), (B, float(np.max(np.abs(got - want))))
        again = run_dev(eng, x_all[:B], 10)
        assert np.array_equal(got.view(np.uint32), again.view(np.uint32))
    # 17 rows: the per-layer kernels again
    got = run_dev(eng, workloads.seeded_input((17,) + tuple(shape)).numpy(), 10)
    assert eng.graph_kernels() > 1 or name == "tiny_mlp"
    eng.close()
    cm.close()


def test_chain_streams_weights_that_do_not_fit(tmp_path):
    """Weight rows that do not fit the CTAs' shared memory (2 x 16 MB here)
    stream from L2 instead of being cached; still the one kernel of the
    forward, still the oracle's values."""
    torch.manual_seed(11)
    m = nn.Sequential(nn.Linear(2048, 2048), nn.ReLU(), nn.Linear(2048, 2048), nn.ReLU(), nn.Linear(2048, 10)).eval()
    cm, eng = engine(m, (2048,), tmp_path)
    x = np.random.default_rng(3).standard_normal((5, 2048)).astype(np.float32)
    got = run_dev(eng, x, 10)
    assert eng.graph_kernels() == 1
    assert np.allclose(got, oracle.run_model(m, x, "fused_ikj"), atol=ATOL, rtol=RTOL)
    eng.close()
    cm.close()


def test_chain_through_public_host_api(tmp_path):
    m = workloads.tiny_mlp()
    cm = compile_model(m, (torch.randn(2, 784),), output_dir=str(tmp_path), autotune=False, enable_fusion=True,
                       kernel_variant="fused_ikj", dynamic_batch=True, max_batch_size=64)
    x = workloads.seeded_input((5, 784)).numpy()
    got = cm.run(x)
    want = oracle.run_model(m, x, "fused_ikj")
    assert np.allclose(got, want, atol=ATOL, rtol=RTOL)
    cm.close()


def test_chain_declines_what_it_cannot_run(tmp_path):
    torch.manual_seed(5)
    # K = 30 is not a multiple of 4: per-layer kernels
    m = nn.Sequential(nn.Linear(30, 20), nn.ReLU(), nn.Linear(20, 6)).eval()
    cm, eng = engine(m, (30,), tmp_path / "a")
    x = np.random.default_rng(0).standard_normal((4, 30)).astype(np.float32)
    got = run_dev(eng, x, 6)
    assert eng.graph_kernels() == 2
    assert np.allclose(got, oracle.run_model(m, x, "fused_ikj"), atol=ATOL, rtol=RTOL)
    eng.close()
    cm.close()
    # an input that is not 16-byte aligned: per-layer kernels, same values
    m2 = workloads.tiny_mlp()
    cm2, eng2 = engine(m2, (784,), tmp_path / "b")
    x2 = workloads.seeded_input((3, 784)).numpy()
    buf = torch.zeros(3 * 784 + 1, dtype=torch.float32, device="cuda")
    buf[1:] = torch.from_numpy(x2).cuda().reshape(-1)
    y2 = torch.empty(30, dtype=torch.float32, device="cuda")
    eng2.run_device(buf.data_ptr() + 4, 3 * 784, y2.data_ptr(), 30, 3, 0)
    torch.cuda.synchronize()
    assert eng2.graph_kernels() > 1
    assert np.allclose(y2.cpu().numpy().reshape(3, 10), oracle.run_model(m2, x2, "fused_ikj"), atol=ATOL, rtol=RTOL)
    eng2.close()
    cm2.close()


@pytest.mark.parametrize("rows", [4, 16])
def test_chain_barrier_timeout_is_reported_and_recoverable(rows, tmp_path):
    """The failure-detection hook makes CTA 0 leave without computing: the
    other CTAs' bounded waits run out (about 2 s) -- at 4 rows for its
    layer-1 values (tagged words), at 16 rows at the first grid barrier --
    they record the error and leave, the last one out resets the counters
    and advances the launch counter, so the next launch's tag differs from
    any word written before; the run returns -5 and the next run is
    correct."""
    m = workloads.tiny_mlp()
    cm, eng = engine(m, (784,), tmp_path)
    x = workloads.seeded_input((rows, 784)).numpy()
    y = np.zeros((rows, 10), np.float32)
    want = oracle.run_model(m, x, "fused_ikj")
    assert eng.run(x, y) == 0
    assert np.allclose(y, want, atol=ATOL, rtol=RTOL)
    lib = _native.lib()
    assert lib.ftb_model_set_fault_injection(eng.handle, 1) == 0
    assert eng.run(x, y) == -5
    assert "exceeded its limit" in _native.last_error()
    assert lib.ftb_model_set_fault_injection(eng.handle, 0) == 0
    y[:] = 0
    assert eng.run(x, y) == 0, _native.last_error()
    assert np.allclose(y, want, atol=ATOL, rtol=RTOL)
    eng.close()
    cm.close()
