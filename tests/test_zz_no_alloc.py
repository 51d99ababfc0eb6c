"""The small-batch GEMM entry point that allocates nothing.

ftb_small_gemm_noalloc exists for callers that may not allocate device memory
where they call in (a plugin inside another engine's execution step, a
latency-critical loop): its split-K scratch is a fixed array inside the
library instead of a context arena.  Called through the C ABI, its output must
match the existing entry point's -- a one-layer model run with
ftb_model_run_device, which uses the same split-K kernel with scratch from the
context arena -- on two calls in a row (the second call finds the previous
call's partial sums in the shared scratch).  Oversized requests are refused
before any launch.

This file is collected last so a failure here leaves every other test run.
"""

import ctypes

import numpy as np
import pytest
import torch
import torch.nn as nn

from forgetune_b200 import _native, compile_model

pytestmark = pytest.mark.gpu

ATOL = RTOL = 1e-4
BIAS, RELU, RESIDUAL = 1, 2, 4


class Layer(nn.Module):
    def __init__(self, k, n, relu, residual):
        super().__init__()
        self.fc = nn.Linear(k, n)
        self.relu = relu
        self.residual = residual

    def forward(self, x):
        y = self.fc(x)
        if self.relu:
            y = torch.relu(y)
        if self.residual:
            y = y + x
        return y


@pytest.mark.parametrize("M,K,N,relu,residual", [(5, 784, 256, True, False), (16, 512, 512, False, True),
                                                 (1, 128, 10, False, False)])
def test_noalloc_matches_existing_entry_point(M, K, N, relu, residual, tmp_path):
    torch.manual_seed(M + K + N)
    model = Layer(K, N, relu, residual).eval()
    cm = compile_model(model, (torch.randn(2, K),), output_dir=str(tmp_path), autotune=False, enable_fusion=True,
                       kernel_variant="fused_ikj", dynamic_batch=True, max_batch_size=64, gpu_kernel="simt",
                       verify=False)
    with open(cm.manifest()["artifacts"]["graph_blob"], "rb") as f:
        eng = _native.EngineModel(f.read())
    dev = torch.device("cuda", torch.cuda.current_device())
    eng.set_devices([dev.index])
    x = torch.from_numpy(np.random.default_rng(N).standard_normal((M, K)).astype(np.float32)).to(dev)
    y_ref = torch.empty((M, N), dtype=torch.float32, device=dev)
    eng.run_device(x.data_ptr(), M * K, y_ref.data_ptr(), M * N, M, 0)
    torch.cuda.synchronize()

    w_kn = model.fc.weight.detach().t().contiguous().to(dev)  # [K, N] row-major
    bias = model.fc.bias.detach().contiguous().to(dev)
    flags = BIAS | (RELU if relu else 0) | (RESIDUAL if residual else 0)
    lib = _native.lib()
    for call in range(2):
        y = torch.full((M, N), float("nan"), dtype=torch.float32, device=dev)
        rc = lib.ftb_small_gemm_noalloc(x.data_ptr(), w_kn.data_ptr(), bias.data_ptr(),
                                        x.data_ptr() if residual else None, y.data_ptr(), M, K, N, flags, None)
        assert rc == 0, _native.last_error()
        torch.cuda.synchronize()
        got, want = y.cpu().numpy(), y_ref.cpu().numpy()
        assert np.allclose(got, want, atol=ATOL, rtol=RTOL), (call, float(np.nanmax(np.abs(got - want))))
    eng.close()
    cm.close()


def test_noalloc_refuses_what_the_scratch_cannot_hold():
    lib = _native.lib()
    p = ctypes.c_void_p(1)  # never dereferenced: the size check comes first
    assert lib.ftb_small_gemm_noalloc(p, p, None, None, p, 17, 64, 64, 0, None) == -2
    assert lib.ftb_small_gemm_noalloc(p, p, None, None, p, 4, 8192, 65536, 0, None) == -2
    assert "scratch" in _native.last_error()
    assert lib.ftb_small_gemm_noalloc(None, p, None, None, p, 4, 64, 64, 0, None) == -1
