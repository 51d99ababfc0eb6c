"""Non-finite inputs.  The reference keeps NaN through ReLU
(tests/correctness/test_audit_regressions.py:685-715, the graph holding only
a ReLU); a NaN in one row of a GEMM input makes that row's outputs NaN and
leaves every other row's bits unchanged, on every kernel path."""

import numpy as np
import pytest
import torch
import torch.nn as nn

from forgetune_b200 import compile_model, workloads

pytestmark = pytest.mark.gpu


class ReluOnly(nn.Module):
    def forward(self, x):
        return torch.relu(x)


@pytest.mark.parametrize("policy", ["auto", "simt", "simt_exact", "tcgen05"])
def test_relu_keeps_nan(policy, tmp_path):
    cm = compile_model(ReluOnly().eval(), (torch.tensor([[1.0, 2.0, 3.0, 4.0]]),), output_dir=str(tmp_path),
                       dynamic_batch=False, autotune=False, gpu_kernel=policy)
    res = cm(np.array([[float("nan"), -1.0, 0.0, 2.5]], dtype=np.float32))
    assert np.isnan(res[0, 0])
    assert res[0, 1] == 0.0 and res[0, 2] == 0.0 and res[0, 3] == 2.5
    cm.close()


@pytest.mark.parametrize("policy,rows", [("auto", 8), ("auto", 300), ("simt", 300), ("simt_exact", 300),
                                         ("tcgen05", 300)])
def test_nan_row_stays_in_its_row(policy, rows, tmp_path):
    m = workloads.tiny_mlp()
    cm = compile_model(m, (workloads.seeded_input((2, 784)),), output_dir=str(tmp_path), autotune=False,
                       kernel_variant="fused_ikj", enable_fusion=True, dynamic_batch=True, max_batch_size=512,
                       gpu_kernel=policy, verify=False)
    x = workloads.seeded_input((rows, 784)).numpy()
    clean = cm.run(x)
    bad = x.copy()
    bad[rows // 2, 17] = np.nan
    out = cm.run(bad)
    assert np.isnan(out[rows // 2]).all()
    keep = np.arange(rows) != rows // 2
    assert np.array_equal(out[keep].view(np.uint32), clean[keep].view(np.uint32))
    cm.close()
