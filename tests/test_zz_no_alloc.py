"""The small-batch GEMM entry point that allocates nothing.

ftb_small_gemm_noalloc exists for callers that may not allocate device memory
where they call in (a plugin inside another engine's execution step, a
latency-critical loop): its split-K scratch is a fixed array inside the
library instead of a context arena.  Called through the C ABI, its output must
match, on two calls in a row (the second call finds the previous call's
partial sums in the shared scratch):

* the CPU oracle's GEMM (bias added after the k sum, NaN-keeping ReLU, then
  the residual), within allclose(1e-4, 1e-4);
* the existing entry point -- the same layer compiled as a model and run
  with ftb_model_run_device, which takes its workspace from the context
  arena -- within the same tolerance.

The second call must not change the device's free memory.  Oversized requests
are refused before any launch.

This file is collected last so a failure here leaves every other test run.
"""

import ctypes

import numpy as np
import pytest
import torch
import torch.nn as nn

from forgetune_b200 import _native, compile_model
from oracle import oracle

pytestmark = pytest.mark.gpu

ATOL = RTOL = 1e-4
BIAS, RELU, RESIDUAL = 1, 2, 4


class Layer(nn.Module):
    def __init__(self, k, n, bias, relu, residual):
        super().__init__()
        self.fc = nn.Linear(k, n, bias=bias)
        self.relu = relu
        self.residual = residual

    def forward(self, x):
        y = self.fc(x)
        if self.relu:
            y = torch.relu(y)
        if self.residual:
            y = y + x
        return y


def oracle_layer(x, w_kn, bias, relu, residual):
    """The reference's node sequence for the layer on the CPU: MATMUL, ADD(bias),
    RELU, ADD(residual), each a separately rounded fp32 step."""
    y = oracle.gemm(x, w_kn, bias, relu=relu, order="bias_last")
    if residual:
        y = (y + x).astype(np.float32)
    return y


@pytest.mark.parametrize("M,K,N,bias,relu,residual", [
    (5, 784, 256, True, True, False),
    (16, 512, 512, True, True, True),     # ReLU and residual together
    (9, 384, 384, True, False, True),
    (1, 128, 10, False, False, False),    # no bias
    (3, 1000, 96, False, True, False),    # no bias, ReLU
])
def test_noalloc_matches_oracle_and_existing_entry_point(M, K, N, bias, relu, residual, tmp_path):
    torch.manual_seed(M + K + N)
    model = Layer(K, N, bias, relu, residual).eval()
    dev = torch.device("cuda", torch.cuda.current_device())
    x_np = np.random.default_rng(N).standard_normal((M, K)).astype(np.float32)
    w_kn_np = model.fc.weight.detach().t().contiguous().numpy()
    b_np = model.fc.bias.detach().numpy() if bias else None
    want = oracle_layer(x_np, w_kn_np, b_np, relu, residual)

    cm = compile_model(model, (torch.randn(2, K),), output_dir=str(tmp_path), autotune=False, enable_fusion=True,
                       kernel_variant="fused_ikj", dynamic_batch=True, max_batch_size=64, gpu_kernel="simt",
                       verify=False)
    with open(cm.manifest()["artifacts"]["graph_blob"], "rb") as f:
        eng = _native.EngineModel(f.read())
    eng.set_devices([dev.index])
    x = torch.from_numpy(x_np).to(dev)
    y_ref = torch.empty((M, N), dtype=torch.float32, device=dev)
    eng.run_device(x.data_ptr(), M * K, y_ref.data_ptr(), M * N, M, 0)  # raises on a non-zero status
    torch.cuda.synchronize()
    existing = y_ref.cpu().numpy()
    assert np.allclose(existing, want, atol=ATOL, rtol=RTOL)

    w_kn = torch.from_numpy(w_kn_np).to(dev)  # [K, N] row-major
    b = torch.from_numpy(b_np).to(dev) if bias else None
    flags = (BIAS if bias else 0) | (RELU if relu else 0) | (RESIDUAL if residual else 0)
    lib = _native.lib()
    ys = [torch.full((M, N), float("nan"), dtype=torch.float32, device=dev) for _ in range(2)]
    torch.cuda.synchronize()
    free_before = None
    for call in range(2):
        if call == 1:
            free_before = torch.cuda.mem_get_info(dev)[0]
        rc = lib.ftb_small_gemm_noalloc(x.data_ptr(), w_kn.data_ptr(), b.data_ptr() if bias else None,
                                        x.data_ptr() if residual else None, ys[call].data_ptr(), M, K, N, flags,
                                        None)
        assert rc == 0, _native.last_error()
        torch.cuda.synchronize()
        if call == 1:
            assert torch.cuda.mem_get_info(dev)[0] == free_before, "a call after the first allocated device memory"
        got = ys[call].cpu().numpy()
        assert np.allclose(got, want, atol=ATOL, rtol=RTOL), (call, float(np.nanmax(np.abs(got - want))))
        assert np.allclose(got, existing, atol=ATOL, rtol=RTOL), (call, float(np.nanmax(np.abs(got - existing))))
    # the shared scratch is fully rewritten: both calls give the same bits
    assert torch.equal(ys[0], ys[1])
    eng.close()
    cm.close()


def test_noalloc_refuses_what_the_scratch_cannot_hold():
    lib = _native.lib()
    p = ctypes.c_void_p(1)  # never dereferenced: the size check comes first
    assert lib.ftb_small_gemm_noalloc(p, p, None, None, p, 17, 64, 64, 0, None) == -2
    assert lib.ftb_small_gemm_noalloc(p, p, None, None, p, 4, 8192, 65536, 0, None) == -2
    assert "scratch" in _native.last_error()
    assert lib.ftb_small_gemm_noalloc(None, p, None, None, p, 4, 64, 64, 0, None) == -1
    assert lib.ftb_small_gemm_noalloc(p, p, None, None, p, 4, 64, 64, BIAS, None) == -1
