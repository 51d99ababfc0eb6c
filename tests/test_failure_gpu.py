"""Failure detection without a GPU fault.

The tensor-core kernels (one SM or an SM pair per tile) bound every mbarrier
wait.  A test hook makes the MMA
thread wait on a barrier that nothing completes: the wait runs out (~2 s), the
kernel raises its abort flag, drains, frees its TMEM and returns; the host
reads the mapped error word and the run returns -5 with a message.  The same
context then runs correctly again.  No trap, bad address or unbounded wait is
used.
"""

import numpy as np
import pytest
import torch
import torch.nn as nn

from forgetune_b200 import _native, compile_model
from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("pair", [1, 2])
def test_tensor_core_wait_timeout_is_reported_and_recoverable(pair, tmp_path):
    """pair=2 runs the SM-pair kernel: the leader CTA's wait runs out, it
    raises its peer's abort flag too, and both CTAs leave together."""
    torch.manual_seed(3)
    m = nn.Sequential(nn.Linear(256, 128), nn.ReLU()).eval()
    cm = compile_model(m, (torch.randn(2, 256),), output_dir=str(tmp_path), autotune=False, enable_fusion=True,
                       kernel_variant="fused_ikj", dynamic_batch=True, max_batch_size=4096,
                       gpu_kernel="tcgen05", verify=False)
    with open(cm.manifest()["artifacts"]["graph_blob"], "rb") as f:
        eng = _native.EngineModel(f.read())
    eng.set_devices([torch.cuda.current_device()])
    eng.set_step_config(0, 0, 0, 0, pair, True)
    x = np.random.default_rng(0).standard_normal((2048, 256)).astype(np.float32)
    y = np.zeros((2048, 128), np.float32)
    assert eng.run(x, y) == 0
    want = oracle.run_model(m, x, "naive_ijk")
    assert np.allclose(y, want, atol=1e-4, rtol=1e-4)

    lib = _native.lib()
    assert lib.ftb_model_set_fault_injection(eng.handle, 1) == 0
    y[:] = 0
    rc = eng.run(x, y)
    assert rc == -5
    assert "exceeded its limit" in _native.last_error()

    assert lib.ftb_model_set_fault_injection(eng.handle, 0) == 0
    assert eng.run(x, y) == 0, _native.last_error()
    assert np.allclose(y, want, atol=1e-4, rtol=1e-4)
    eng.close()
    cm.close()


@pytest.mark.parametrize("pair,rows", [(4, 3000), (5, 2048), (5, 20000)])
def test_two_layer_kernel_wait_timeout_is_reported_and_recoverable(pair, rows, tmp_path):
    """The two-layer kernel (both layers and the head in one launch, the
    hidden layer in tensor memory), unsplit and split over teams of pairs:
    its MMA thread's wait runs out, every role of both CTAs leaves through
    its own bounded waits (a team owner also stops waiting for its helpers;
    at 20000 rows the full rounds run unsplit and the last round by teams),
    the run returns -5, and the same context then computes correctly again."""
    torch.manual_seed(4)
    m = nn.Sequential(nn.Linear(256, 256), nn.ReLU(), nn.Linear(256, 128), nn.ReLU(), nn.Linear(128, 10)).eval()
    cm = compile_model(m, (torch.randn(2, 256),), output_dir=str(tmp_path), autotune=False, enable_fusion=True,
                       kernel_variant="fused_ikj", dynamic_batch=True, max_batch_size=20000,
                       gpu_kernel="tcgen05", verify=False)
    with open(cm.manifest()["artifacts"]["graph_blob"], "rb") as f:
        eng = _native.EngineModel(f.read())
    eng.set_devices([torch.cuda.current_device()])
    assert eng.describe()["steps"][0]["mlp_step"] == 1
    eng.set_step_config(0, 0, 0, 0, pair, True)  # pair 5 at 8 tiles: layer 1 split over teams of 2 pairs
    x = np.random.default_rng(1).standard_normal((rows, 256)).astype(np.float32)
    y = np.zeros((rows, 10), np.float32)
    assert eng.run(x, y) == 0
    want = oracle.run_model(m, x, "naive_ijk")
    assert np.allclose(y, want, atol=1e-4, rtol=1e-4)

    lib = _native.lib()
    assert lib.ftb_model_set_fault_injection(eng.handle, 1) == 0
    y[:] = 0
    assert eng.run(x, y) == -5
    assert "exceeded its limit" in _native.last_error()

    assert lib.ftb_model_set_fault_injection(eng.handle, 0) == 0
    assert eng.run(x, y) == 0, _native.last_error()
    assert np.allclose(y, want, atol=1e-4, rtol=1e-4)
    eng.close()
    cm.close()


def test_convolution_wait_timeout_is_reported_and_recoverable(tmp_path):
    """The implicit-GEMM convolution's MMA thread waits on a barrier nothing
    completes: the wait runs out, the gather, producer and epilogue warps
    leave through their bounded waits, the run returns -5, and the same
    context then computes correctly again."""
    torch.manual_seed(6)
    m = nn.Sequential(nn.Conv2d(8, 64, 3, padding=1), nn.ReLU()).eval()
    cm = compile_model(m, (torch.randn(2, 8, 16, 16),), output_dir=str(tmp_path), autotune=False,
                       enable_fusion=True, kernel_variant="fused_ikj", dynamic_batch=True, max_batch_size=64,
                       gpu_kernel="tcgen05", verify=False)
    with open(cm.manifest()["artifacts"]["graph_blob"], "rb") as f:
        eng = _native.EngineModel(f.read())
    eng.set_devices([torch.cuda.current_device()])
    x = np.random.default_rng(2).standard_normal((16, 8, 16, 16)).astype(np.float32)
    y = np.zeros((16, 64, 16, 16), np.float32)
    want = oracle.run_model(m, x, "fused_ikj")
    assert eng.run(x, y) == 0
    assert np.allclose(y, want, atol=1e-4, rtol=1e-4)
    lib = _native.lib()
    assert lib.ftb_model_set_fault_injection(eng.handle, 1) == 0
    assert eng.run(x, y) == -5
    assert "exceeded its limit" in _native.last_error()
    assert lib.ftb_model_set_fault_injection(eng.handle, 0) == 0
    y[:] = 0
    assert eng.run(x, y) == 0, _native.last_error()
    assert np.allclose(y, want, atol=1e-4, rtol=1e-4)
    eng.close()
    cm.close()
