"""The narrow-N GEMM (N <= 16 columns, more than 16 rows, non-exact
policies): every N from 1 to 16 class, K across the 256-row W chunks, both
bias orders, and both forms -- one warp per 32 rows when the row blocks fill
the SMs, eight warps splitting K over 32 rows when they do not; against the
oracle with the reference's tolerance, bitwise run to run."""

import numpy as np
import pytest
import torch
import torch.nn as nn

from forgetune_b200 import compile_model
from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,K,N", [(17, 7, 1), (1000, 128, 10), (5000, 600, 16), (333, 300, 3), (64, 33, 12),
                                   (1024, 512, 10), (256, 128, 10), (40, 4000, 4), (19000, 200, 10)])
@pytest.mark.parametrize("variant", ["fused_ikj", "naive_ijk"])
def test_narrow_gemm_matches_oracle(M, K, N, variant, tmp_path):
    torch.manual_seed(M + N)
    m = nn.Sequential(nn.Linear(K, N), nn.ReLU()).eval()
    cm = compile_model(m, (torch.randn(2, K),), output_dir=str(tmp_path), autotune=False, enable_fusion=True,
                       kernel_variant=variant, dynamic_batch=True, max_batch_size=M, gpu_kernel="simt",
                       verify=False)
    x = np.random.default_rng(K).standard_normal((M, K)).astype(np.float32)
    got = cm.run(x)
    want = oracle.run_model(m, x, variant)
    assert np.allclose(got, want, atol=1e-4, rtol=1e-4), float(np.max(np.abs(got - want)))
    assert np.array_equal(got.view(np.uint32), cm.run(x).view(np.uint32))
    cm.close()
