"""Split-K GEMM for small batches (M <= 16): ragged K and N, every epilogue
form, against the CPU oracle with the reference tolerance, and bitwise run to
run (the slice partials are summed in a fixed order by whichever CTA finishes
last)."""

import numpy as np
import pytest
import torch
import torch.nn as nn

from forgetune_b200 import compile_model
from oracle import oracle

pytestmark = pytest.mark.gpu


class Lin(nn.Module):
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


SHAPES = [(1, 784, 256, True, False), (3, 5, 10, False, False), (8, 8192, 8192, True, False),
          (9, 128, 10, False, False), (16, 512, 512, False, True), (1, 1, 1, False, False),
          (2, 100, 65, True, False), (16, 4096, 63, False, False), (5, 2048, 2048, False, True)]


@pytest.mark.parametrize("M,K,N,relu,residual", SHAPES)
def test_splitk_matches_oracle(M, K, N, relu, residual, tmp_path):
    torch.manual_seed(K * 7 + N)
    m = Lin(K, N, relu, residual).eval()
    cm = compile_model(m, (torch.randn(2, K),), output_dir=str(tmp_path), autotune=False, enable_fusion=True,
                       kernel_variant="fused_ikj", dynamic_batch=True, max_batch_size=64,
                       max_workspace_bytes=4 << 30, gpu_kernel="simt", verify=False)
    x = np.random.default_rng(M * 131 + K).standard_normal((M, K)).astype(np.float32)
    got = cm.run(x)
    want = oracle.gemm(x, m.fc.weight.detach().numpy().T.copy(), m.fc.bias.detach().numpy(), relu=relu,
                       order="bias_last")
    if residual:
        want = oracle.add(want, x)
    assert np.allclose(got, want, atol=1e-4, rtol=1e-4), float(np.max(np.abs(got - want)))
    for _ in range(3):
        assert np.array_equal(got.view(np.uint32), cm.run(x).view(np.uint32))
    cm.close()
