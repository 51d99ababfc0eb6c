"""The five forward-pass workloads this backend is measured and checked on.

Each builder seeds torch's CPU generator with 0 and constructs the layers in
declaration order with PyTorch's default ``nn.Linear`` / ``nn.Conv2d``
initialisation, so the weights are a pure function of the torch version.
Inputs are N(0, 1) float32 drawn from a separate CPU generator seeded with 1
(``torch.randn(shape, generator=Generator().manual_seed(1))``); a prefix of a
larger draw equals a smaller draw, so B=64 rows of the dynamic tiny MLP are
the first 64 rows of its B=65536 input.

The wide MLP's input (262144 x 4096, 4.3 GB) is generated on the device per
shard by the counter-based normal generator in ``forgetune_b200.philox``
instead, keyed by the global element index so that it does not depend on how
the batch is split across GPUs.
"""

from __future__ import annotations

import torch
import torch.nn as nn

__all__ = [
    "ResidualBlock",
    "tiny_mlp",
    "residual_mlp",
    "small_cnn",
    "wide_mlp",
    "op_mix",
    "OpMix",
    "seeded_input",
    "WORKLOADS",
]


class ResidualBlock(nn.Module):
    """y = x + fc2(relu(fc1(x))) with two Linear(width, width) layers."""

    def __init__(self, width: int):
        super().__init__()
        self.fc1 = nn.Linear(width, width)
        self.fc2 = nn.Linear(width, width)

    def forward(self, x):
        return x + self.fc2(torch.relu(self.fc1(x)))


def tiny_mlp() -> nn.Module:
    """Linear(784,256)+ReLU, Linear(256,128)+ReLU, Linear(128,10)."""
    torch.manual_seed(0)
    return nn.Sequential(
        nn.Linear(784, 256), nn.ReLU(),
        nn.Linear(256, 128), nn.ReLU(),
        nn.Linear(128, 10),
    ).eval()


def residual_mlp() -> nn.Module:
    """Linear(512,512) stem, 4 residual blocks of width 512, Linear(512,10) head."""
    torch.manual_seed(0)
    return nn.Sequential(
        nn.Linear(512, 512),
        ResidualBlock(512), ResidualBlock(512), ResidualBlock(512), ResidualBlock(512),
        nn.Linear(512, 10),
    ).eval()


def small_cnn() -> nn.Module:
    """NCHW 3x32x32 -> conv(32,s1) -> conv(64,s2) -> conv(64,s2) -> flatten -> 128 -> 10."""
    torch.manual_seed(0)
    return nn.Sequential(
        nn.Conv2d(3, 32, 3, stride=1, padding=1), nn.ReLU(),
        nn.Conv2d(32, 64, 3, stride=2, padding=1), nn.ReLU(),
        nn.Conv2d(64, 64, 3, stride=2, padding=1), nn.ReLU(),
        nn.Flatten(),
        nn.Linear(4096, 128), nn.ReLU(),
        nn.Linear(128, 10),
    ).eval()


def wide_mlp() -> nn.Module:
    """Linear(4096,8192)+ReLU, Linear(8192,8192)+ReLU, Linear(8192,4096)."""
    torch.manual_seed(0)
    return nn.Sequential(
        nn.Linear(4096, 8192), nn.ReLU(),
        nn.Linear(8192, 8192), nn.ReLU(),
        nn.Linear(8192, 4096),
    ).eval()


class OpMix(nn.Module):
    """Every un-fused node form of the reference's code generator in one
    small NCHW model (src/codegen.cpp:835-958): a convolution without ReLU,
    ADD and MUL with a channel operand [C,1,1] on NCHW, ADD with a [1,N] row,
    MUL with an [N] row, SIGMOID, TANH, MUL and ADD of same-shape tensors,
    FLATTEN and Linear layers without a fused ReLU.  Input [B, 3, 8, 8]."""

    def __init__(self):
        super().__init__()
        self.conv = nn.Conv2d(3, 8, 3, padding=1)
        self.ch_shift = nn.Parameter(0.1 * torch.randn(8, 1, 1))
        self.ch_scale = nn.Parameter(0.5 + torch.rand(8, 1, 1))
        self.fc1 = nn.Linear(512, 64)
        self.col_scale = nn.Parameter(0.5 + torch.rand(64))
        self.row_shift = nn.Parameter(0.1 * torch.randn(1, 64))
        self.fc2 = nn.Linear(64, 64)
        self.head = nn.Linear(64, 10)

    def forward(self, x):
        h = self.conv(x) + self.ch_shift
        h = torch.relu(h * self.ch_scale)
        h = torch.flatten(h, 1)
        h = self.fc1(h) * self.col_scale
        h = h + self.row_shift
        a = torch.sigmoid(h)
        b = torch.tanh(self.fc2(h))
        h = a * b + a
        return self.head(h)


def op_mix() -> nn.Module:
    torch.manual_seed(0)
    return OpMix().eval()


def seeded_input(shape, seed: int = 1) -> torch.Tensor:
    """N(0,1) float32 CPU tensor drawn from ``Generator().manual_seed(seed)``."""
    g = torch.Generator().manual_seed(seed)
    return torch.randn(tuple(shape), generator=g, dtype=torch.float32)


# name -> (builder, per-sample input shape, batch the workload is quoted at)
WORKLOADS = {
    "tiny_mlp": (tiny_mlp, (784,), 64),
    "tiny_mlp_dynamic": (tiny_mlp, (784,), 65536),
    "residual_mlp": (residual_mlp, (512,), 1024),
    "small_cnn": (small_cnn, (3, 32, 32), 256),
    "wide_mlp": (wide_mlp, (4096,), 262144),
    # op coverage (not a measured workload): the reference's elementwise forms
    "op_mix": (op_mix, (3, 8, 8), 64),
}
