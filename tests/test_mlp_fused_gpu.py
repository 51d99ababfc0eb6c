"""Two consecutive Linear layers (and a small head after them) computed by one
tcgen05 kernel on SM pairs, the first layer's output kept in tensor memory
and read back as the second layer's A operand.  Unsplit (pair 4), the kernel
performs the same operations in the same order as two separate SM-pair
launches, so the outputs must agree bit for bit.  With few tiles the shape
rule (or pair 5) splits layer 1's k-blocks over a team of pairs per tile:
deterministic run to run, a different association of the k sums.  Every
form is held to the reference's tolerance against the CPU oracle."""

import numpy as np
import pytest
import torch
import torch.nn as nn

from forgetune_b200 import _native, compile_model
from oracle import oracle

pytestmark = pytest.mark.gpu

CASES = [
    # M, K1, N1, N2, head, relu1, relu2
    (20000, 784, 256, 128, 10, True, True),   # the tiny MLP's layers, 79 tiles over the pairs
    (17, 784, 256, 128, 10, True, True),      # one partial tile
    (300, 100, 200, 64, 0, True, False),      # no head: layer 2's output stored; N1 = 200 (ragged chunk)
    (1000, 256, 144, 100, 7, False, True),    # odd count of layer-2 k-blocks, N2 not a multiple of 16
    (5000, 64, 256, 128, 16, True, True),
    (777, 96, 160, 70, 0, False, False),      # no head, rows of 70 floats: the transposing store epilogue
]


def _model(K1, N1, N2, head, relu1, relu2):
    layers = [nn.Linear(K1, N1)] + ([nn.ReLU()] if relu1 else []) + [nn.Linear(N1, N2)]
    layers += [nn.ReLU()] if relu2 else []
    layers += [nn.Linear(N2, head)] if head else []
    return nn.Sequential(*layers).eval()


def _run_device(eng, x, out_cols):
    dev = torch.cuda.current_device()
    xd = torch.from_numpy(x).to(dev)
    yd = torch.zeros((x.shape[0], out_cols), dtype=torch.float32, device=dev)
    eng.run_device(xd.data_ptr(), xd.numel(), yd.data_ptr(), yd.numel(), x.shape[0],
                   torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return yd.cpu().numpy(), eng.graph_kernels()


@pytest.mark.parametrize("M,K1,N1,N2,head,relu1,relu2", CASES)
def test_two_layers_in_one_kernel_match_two_launches(M, K1, N1, N2, head, relu1, relu2, tmp_path):
    torch.manual_seed(M + N1 + N2)
    m = _model(K1, N1, N2, head, relu1, relu2)
    cm = compile_model(m, (torch.randn(2, K1),), output_dir=str(tmp_path), autotune=False, enable_fusion=True,
                       kernel_variant="fused_ikj", dynamic_batch=True, max_batch_size=M,
                       max_workspace_bytes=8 << 30, gpu_kernel="tcgen05", verify=False)
    with open(cm.manifest()["artifacts"]["graph_blob"], "rb") as f:
        eng = _native.EngineModel(f.read())
    eng.set_devices([torch.cuda.current_device()])
    steps = eng.describe()["steps"]
    assert steps[0]["mlp_step"] == 1 and steps[1]["mlp_of"] == 0, steps
    out_cols = head or N2
    x = np.random.default_rng(M).standard_normal((M, K1)).astype(np.float32)
    want = oracle.run_model(m, x, "naive_ijk")

    # by shape (a team split when the tiles are few)
    shaped, k_shaped = _run_device(eng, x, out_cols)
    assert k_shaped == 1, "expected the whole launch list as one kernel, got %d" % k_shaped
    assert np.allclose(shaped, want, atol=1e-4, rtol=1e-4), float(np.max(np.abs(shaped - want)))

    # asked for explicitly without a split (pair 4)
    eng.set_step_config(0, 0, 0, 0, 4, True)
    fused, k_fused = _run_device(eng, x, out_cols)
    assert k_fused == 1
    assert np.allclose(fused, want, atol=1e-4, rtol=1e-4), float(np.max(np.abs(fused - want)))

    # the same layers as separate SM-pair launches (an explicit tile
    # configuration turns the two-layer kernel off): the same bits
    eng.set_step_config(0, 0, 0, 0, 2, True)
    eng.set_step_config(1, 0, 0, 0, 2, True)
    apart, k_apart = _run_device(eng, x, out_cols)
    assert k_apart == 2, k_apart
    assert np.array_equal(fused.view(np.uint32), apart.view(np.uint32)), \
        float(np.max(np.abs(fused - apart)))

    # the team split asked for (pair 5): within tolerance, the same bits run
    # to run, and the shape rule's result (which splits the same tiles: all
    # of them when they are few, a sparse last round when they are many)
    eng.set_step_config(0, 0, 0, 0, 5, True)
    eng.set_step_config(1, 0, 0, 0, 0, True)
    team, k_team = _run_device(eng, x, out_cols)
    assert k_team == 1
    assert np.allclose(team, want, atol=1e-4, rtol=1e-4), float(np.max(np.abs(team - want)))
    team2, _ = _run_device(eng, x, out_cols)
    assert np.array_equal(team.view(np.uint32), team2.view(np.uint32))
    assert np.array_equal(team.view(np.uint32), shaped.view(np.uint32))
    eng.close()
    cm.close()


@pytest.mark.parametrize("M", [1, 64, 300, 4096, 8192, 9472, 20000, 65536])
def test_team_split_on_the_tiny_mlp_layers(M, tmp_path):
    """The tiny MLP's shapes at the row counts where layer 1 splits over
    teams of two pairs: every tile up to 37 tiles; at 79 and 256 tiles the
    last round (5 and 34 tiles on 74 pairs) while the full rounds run
    unsplit.  The oracle's values within tolerance, the same bits run to
    run."""
    torch.manual_seed(7)
    m = _model(784, 256, 128, 10, True, True)
    cm = compile_model(m, (torch.randn(2, 784),), output_dir=str(tmp_path), autotune=False, enable_fusion=True,
                       kernel_variant="fused_ikj", dynamic_batch=True, max_batch_size=max(M, 17),
                       gpu_kernel="tcgen05", verify=False)
    with open(cm.manifest()["artifacts"]["graph_blob"], "rb") as f:
        eng = _native.EngineModel(f.read())
    eng.set_devices([torch.cuda.current_device()])
    eng.set_step_config(0, 0, 0, 0, 5, True)
    x = np.random.default_rng(M).standard_normal((M, 784)).astype(np.float32)
    want = oracle.run_model(m, x, "fused_ikj")
    got, k = _run_device(eng, x, 10)
    assert k == 1
    assert np.allclose(got, want, atol=1e-4, rtol=1e-4), float(np.max(np.abs(got - want)))
    again, _ = _run_device(eng, x, 10)
    assert np.array_equal(got.view(np.uint32), again.view(np.uint32))
    eng.close()
    cm.close()
