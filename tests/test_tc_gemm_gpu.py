"""The tcgen05 3xTF32 GEMM on ragged shapes: M not a multiple of the 128-row
tile, K not a multiple of the 32-wide k-block, N not a multiple of the tile
width or of 4, each epilogue form; against the CPU oracle with the
reference's tolerance, and bitwise run to run."""

import numpy as np
import pytest
import torch
import torch.nn as nn

from forgetune_b200 import compile_model
from oracle import oracle

pytestmark = pytest.mark.gpu


class Block(nn.Module):
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


SHAPES = [
    # M, K, N, relu, residual
    (1000, 784, 256, True, False),
    (257, 96, 200, False, False),
    (4097, 512, 512, False, True),
    (130, 36, 64, True, False),
    (2048, 1024, 50, False, False),
    (300, 128, 384, True, False),
    (65536, 784, 256, True, False),
]


@pytest.mark.parametrize("M,K,N,relu,residual", SHAPES)
def test_tcgen05_matches_oracle(M, K, N, relu, residual, tmp_path):
    if residual:
        assert K == N
    torch.manual_seed(M + K + N)
    m = Block(K, N, relu, residual).eval()
    cm = compile_model(m, (torch.randn(2, K),), output_dir=str(tmp_path), autotune=False, enable_fusion=True,
                       kernel_variant="fused_ikj", dynamic_batch=True, max_batch_size=max(M, 2),
                       max_workspace_bytes=8 << 30, gpu_kernel="tcgen05", verify=False)
    steps = cm.plan()["steps"]
    assert steps[0]["K"] == K and steps[0]["N"] == N
    x = np.random.default_rng(M).standard_normal((M, K)).astype(np.float32)
    got = cm.run(x)
    w = m.fc.weight.detach().numpy().T.copy()
    want = oracle.gemm(x, w, m.fc.bias.detach().numpy(), relu=relu, order="bias_last")
    if residual:
        want = oracle.add(want, x)
    assert np.allclose(got, want, atol=1e-4, rtol=1e-4), float(np.max(np.abs(got - want)))
    again = cm.run(x)
    assert np.array_equal(got.view(np.uint32), again.view(np.uint32))
    cm.close()


@pytest.mark.parametrize("M,K,H,N2", [(3000, 96, 128, 7), (65536, 256, 128, 10), (1500, 64, 256, 16),
                                      (2000, 128, 200, 3), (1024, 128, 320, 10)])
def test_fused_small_head_matches_oracle(M, K, H, N2, tmp_path):
    """Linear+ReLU followed by a Linear with <= 16 outputs: the head is
    computed in the tensor-core epilogue (the hidden layer is never stored)
    when the hidden width fits one tile, and as its own step otherwise."""
    torch.manual_seed(M + H)
    m = nn.Sequential(nn.Linear(K, H), nn.ReLU(), nn.Linear(H, N2)).eval()
    cm = compile_model(m, (torch.randn(2, K),), output_dir=str(tmp_path), autotune=False, enable_fusion=True,
                       kernel_variant="fused_ikj", dynamic_batch=True, max_batch_size=M,
                       max_workspace_bytes=8 << 30, gpu_kernel="tcgen05", verify=False)
    x = np.random.default_rng(H).standard_normal((M, K)).astype(np.float32)
    got = cm.run(x)
    want = oracle.run_model(m, x, "naive_ijk")
    assert got.shape == (M, N2)
    assert np.allclose(got, want, atol=1e-4, rtol=1e-4), float(np.max(np.abs(got - want)))
    assert np.array_equal(got.view(np.uint32), cm.run(x).view(np.uint32))
    cm.close()


# (tile width, k-block, 128-row halves on one SM, 2 = 256-row tiles on an SM pair)
TILE_CONFIGS = [(64, 16, 1, 1), (128, 16, 1, 1), (256, 16, 1, 1), (64, 32, 1, 1), (128, 32, 1, 1), (256, 32, 1, 1),
                (64, 16, 2, 1), (128, 16, 2, 1), (64, 32, 2, 1), (128, 32, 2, 1),
                (128, 16, 1, 2), (256, 16, 1, 2), (128, 32, 1, 2), (256, 32, 1, 2)]


@pytest.mark.parametrize("M,K,N", [(3000, 784, 256), (700, 96, 130), (2300, 512, 64), (129, 64, 300)])
def test_every_tile_configuration_agrees(M, K, N, tmp_path):
    """Tile width, k-block, 128/256-row tiles and one SM or an SM pair per
    tile change only the schedule: each output element is the same sequence
    of MMAs, so all configurations give the same bits, within tolerance of
    the oracle."""
    from forgetune_b200 import _native
    torch.manual_seed(M)
    m = Block(K, N, True, False).eval()
    cm = compile_model(m, (torch.randn(2, K),), output_dir=str(tmp_path), autotune=False, enable_fusion=True,
                       kernel_variant="fused_ikj", dynamic_batch=True, max_batch_size=M,
                       gpu_kernel="tcgen05", verify=False)
    with open(cm.manifest()["artifacts"]["graph_blob"], "rb") as f:
        eng = _native.EngineModel(f.read())
    eng.set_devices([torch.cuda.current_device()])
    x = np.random.default_rng(K).standard_normal((M, K)).astype(np.float32)
    want = oracle.gemm(x, m.fc.weight.detach().numpy().T.copy(), m.fc.bias.detach().numpy(), relu=True,
                       order="bias_last")
    first = None
    for bn, bk, mh, pair in TILE_CONFIGS:
        eng.set_step_config(0, bn, bk, mh, pair, True)
        y = np.zeros((M, N), np.float32)
        assert eng.run(x, y) == 0, _native.last_error()
        assert np.allclose(y, want, atol=1e-4, rtol=1e-4), (bn, bk, mh, pair, float(np.max(np.abs(y - want))))
        if first is None:
            first = y.copy()
        assert np.array_equal(y.view(np.uint32), first.view(np.uint32)), (bn, bk, mh, pair)
    eng.close()
    cm.close()


@pytest.mark.parametrize("M,K,H,N2", [(3000, 96, 128, 7), (65536, 256, 128, 10), (1500, 64, 256, 16)])
def test_fused_head_on_sm_pairs_agrees(M, K, H, N2, tmp_path):
    """The small head fused into the epilogue of SM-pair tiles gives the
    same bits as on one-SM tiles."""
    from forgetune_b200 import _native
    torch.manual_seed(M + H)
    m = nn.Sequential(nn.Linear(K, H), nn.ReLU(), nn.Linear(H, N2)).eval()
    cm = compile_model(m, (torch.randn(2, K),), output_dir=str(tmp_path), autotune=False, enable_fusion=True,
                       kernel_variant="fused_ikj", dynamic_batch=True, max_batch_size=M,
                       max_workspace_bytes=8 << 30, gpu_kernel="tcgen05", verify=False)
    with open(cm.manifest()["artifacts"]["graph_blob"], "rb") as f:
        eng = _native.EngineModel(f.read())
    eng.set_devices([torch.cuda.current_device()])
    x = np.random.default_rng(H).standard_normal((M, K)).astype(np.float32)
    want = oracle.run_model(m, x, "naive_ijk")
    outs = []
    for pair in (1, 2):
        eng.set_step_config(0, 0, 0, 0, pair, True)
        y = np.zeros((M, N2), np.float32)
        assert eng.run(x, y) == 0, _native.last_error()
        assert np.allclose(y, want, atol=1e-4, rtol=1e-4), (pair, float(np.max(np.abs(y - want))))
        outs.append(y)
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
    eng.close()
    cm.close()


CONVS = [
    # B, Cin, H, W, Cout, k, stride, pad, dilation, relu
    (256, 3, 32, 32, 32, 3, 1, 1, 1, True),      # the CNN's first layer: K = 27 padded to 32
    (256, 32, 32, 32, 64, 3, 2, 1, 1, True),     # second: stride 2
    (64, 64, 8, 8, 64, 3, 2, 1, 1, False),
    (7, 5, 13, 11, 40, 3, 1, 2, 2, True),        # dilation 2, Cout not a multiple of 32, odd sizes
    (3, 8, 9, 9, 48, 1, 1, 0, 1, False),         # 1x1
    (100, 16, 64, 64, 32, 3, 1, 1, 1, True),     # 409600 pixels: 3200 tiles over the SMs
    (5, 12, 10, 10, 96, 3, 1, 1, 1, True),       # 128-channel tiles, 96 in range
    (2, 4, 15, 17, 300, 5, 2, 2, 1, False),      # 256-channel tiles: two column tiles, the second partial
]


@pytest.mark.parametrize("B,Cin,H,W,Cout,k,stride,pad,dil,relu", CONVS)
def test_tcgen05_convolution_matches_oracle(B, Cin, H, W, Cout, k, stride, pad, dil, relu, tmp_path):
    """Convolution as an implicit GEMM on the tensor cores (the input gathered
    per k-block, NCHW stores from the epilogue), against the oracle's direct
    convolution with the reference's tolerance, bitwise run to run."""
    torch.manual_seed(Cin * 100 + Cout)
    layers = [nn.Conv2d(Cin, Cout, k, stride=stride, padding=pad, dilation=dil)]
    if relu:
        layers.append(nn.ReLU())
    m = nn.Sequential(*layers).eval()
    cm = compile_model(m, (torch.randn(2, Cin, H, W),), output_dir=str(tmp_path), autotune=False,
                       enable_fusion=True, kernel_variant="fused_ikj", dynamic_batch=True, max_batch_size=B,
                       max_workspace_bytes=8 << 30, gpu_kernel="tcgen05", verify=False)
    x = np.random.default_rng(B + Cout).standard_normal((B, Cin, H, W)).astype(np.float32)
    got = cm.run(x)
    conv = m[0]
    want = oracle.conv2d(x, conv.weight.detach().numpy(), conv.bias.detach().numpy(), (stride, stride), (pad, pad),
                         (dil, dil), relu=relu)
    assert got.shape == want.shape
    assert np.allclose(got, want, atol=1e-4, rtol=1e-4), float(np.max(np.abs(got - want)))
    assert np.array_equal(got.view(np.uint32), cm.run(x).view(np.uint32))
    cm.close()


@pytest.mark.parametrize("M,K,N,relu,residual", [(256, 4096, 128, True, False), (1024, 512, 512, False, True),
                                                 (300, 2048, 256, True, False), (17, 1024, 132, False, False)])
@pytest.mark.parametrize("pair", [0, 3])
def test_split_k_matches_oracle(M, K, N, relu, residual, pair, tmp_path):
    """Few tiles and a long K: the SM-pair kernel splits K into ranges whose
    partial sums a reduction adds in a fixed order (shape rules, pair=0, and
    the explicit choice, pair=3); within tolerance of the oracle, bitwise run
    to run."""
    from forgetune_b200 import _native
    torch.manual_seed(M + K)
    m = Block(K, N, relu, residual).eval() if not residual else Block(K, K, relu, True).eval()
    n_out = K if residual else N
    cm = compile_model(m, (torch.randn(2, K),), output_dir=str(tmp_path), autotune=False, enable_fusion=True,
                       kernel_variant="fused_ikj", dynamic_batch=True, max_batch_size=max(M, 2),
                       gpu_kernel="tcgen05", verify=False)
    with open(cm.manifest()["artifacts"]["graph_blob"], "rb") as f:
        eng = _native.EngineModel(f.read())
    eng.set_devices([torch.cuda.current_device()])
    eng.set_step_config(0, 0, 0, 0, pair, True)
    x = np.random.default_rng(K).standard_normal((M, K)).astype(np.float32)
    y = np.zeros((M, n_out), np.float32)
    assert eng.run(x, y) == 0, _native.last_error()
    want = oracle.gemm(x, m.fc.weight.detach().numpy().T.copy(), m.fc.bias.detach().numpy(), relu=relu,
                       order="bias_last")
    if residual:
        want = oracle.add(want, x)
    assert np.allclose(y, want, atol=1e-4, rtol=1e-4), float(np.max(np.abs(y - want)))
    y2 = np.zeros_like(y)
    assert eng.run(x, y2) == 0
    assert np.array_equal(y.view(np.uint32), y2.view(np.uint32))
    eng.close()
    cm.close()
