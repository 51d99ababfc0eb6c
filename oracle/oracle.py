"""CPU oracle driver -- TEST INFRASTRUCTURE ONLY.

Walks a supported ``torch.nn`` model and evaluates it with the C restatement
in ``forward_oracle.c``, applying the node sequence the reference produces for
it: the export frontend lowers Linear to MATMUL(x, W^T) + ADD(bias)
(python/forgetune/export_frontend.py:224-297) and Conv2d to CONV2D
(:622-698); the fusion pass then turns MATMUL->ADD->RELU into
FUSED_MATMUL_ADD_RELU and CONV2D->RELU into FUSED_CONV2D_RELU when the
intermediates have a single use (src/fusion.cpp:6-131).  The result is the
reference runtime's output, bit for bit, for the ``fused_ikj`` and
``naive_ijk`` variants.

Only tests, the smoke check and the benchmark's CPU-baseline leg may import
this module.  It is never part of the product path.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
import sys
from typing import List, Tuple

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
SRC_PATH = os.path.join(HERE, "forward_oracle.c")

_lib = None

_F = ctypes.POINTER(ctypes.c_float)


def build(force: bool = False) -> str:
    """Compile forward_oracle.c into liboracle.so beside it (gcc, no FMA contraction)."""
    if force or not os.path.isfile(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(SRC_PATH):
        tmp = LIB_PATH + ".tmp%d" % os.getpid()
        subprocess.check_call([
            "gcc", "-O2", "-fPIC", "-shared", "-std=c11", "-ffp-contract=off",
            "-fno-signed-zeros", "-o", tmp, SRC_PATH, "-lm",
        ])
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(LIB_PATH)
        i64, vp = ctypes.c_int64, ctypes.c_void_p
        for name in ("ora_gemm_bias_first", "ora_gemm_bias_last"):
            fn = getattr(L, name)
            fn.argtypes = [i64, i64, i64, vp, vp, vp, ctypes.c_int, ctypes.c_int, vp]
            fn.restype = None
        L.ora_add.argtypes = [i64, vp, vp, vp]
        L.ora_add_row.argtypes = [i64, i64, vp, vp, vp]
        L.ora_add_channel.argtypes = [i64, i64, i64, vp, vp, vp]
        L.ora_relu.argtypes = [i64, vp, vp]
        L.ora_mul.argtypes = [i64, vp, vp, vp]
        L.ora_mul_row.argtypes = [i64, i64, vp, vp, vp]
        L.ora_mul_channel.argtypes = [i64, i64, i64, vp, vp, vp]
        L.ora_sigmoid.argtypes = [i64, vp, vp]
        L.ora_tanh.argtypes = [i64, vp, vp]
        L.ora_conv2d.argtypes = [i64] * 13 + [vp, vp, vp, ctypes.c_int, vp]
        L.ora_conv2d.restype = ctypes.c_int
        L.ora_philox_blocks.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, vp]
        L.ora_philox_normal.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, vp]
        _lib = L
    return _lib


def _p(a: np.ndarray):
    return a.ctypes.data


def _f32(a) -> np.ndarray:
    if hasattr(a, "detach"):
        a = a.detach().cpu().numpy()
    return np.ascontiguousarray(a, dtype=np.float32)


# --------------------------------------------------------------------------
# single ops
# --------------------------------------------------------------------------

def gemm(x: np.ndarray, w_kn: np.ndarray, bias=None, relu=False, order="bias_first") -> np.ndarray:
    """y = (relu?)(x @ w_kn + bias) in the reference's bias-first or bias-last order."""
    x = _f32(x)
    w_kn = _f32(w_kn)
    M, K = x.shape
    K2, N = w_kn.shape
    assert K == K2
    y = np.empty((M, N), dtype=np.float32)
    b = _f32(bias) if bias is not None else None
    bias_rows = int(b is not None and b.ndim == 2 and b.shape[0] > 1)
    fn = lib().ora_gemm_bias_first if order == "bias_first" else lib().ora_gemm_bias_last
    fn(M, K, N, _p(x), _p(w_kn), _p(b) if b is not None else None, bias_rows, int(relu), _p(y))
    return y


def conv2d(x, w, bias, stride, padding, dilation, relu=False) -> np.ndarray:
    x = _f32(x)
    w = _f32(w)
    B, Cin, H, W = x.shape
    Cout, Cin2, Kh, Kw = w.shape
    assert Cin == Cin2
    sh, sw = stride
    ph, pw = padding
    dh, dw = dilation
    Ho = (H + 2 * ph - (dh * (Kh - 1) + 1)) // sh + 1
    Wo = (W + 2 * pw - (dw * (Kw - 1) + 1)) // sw + 1
    y = np.empty((B, Cout, Ho, Wo), dtype=np.float32)
    b = _f32(bias) if bias is not None else None
    rc = lib().ora_conv2d(B, Cin, H, W, Cout, Kh, Kw, sh, sw, ph, pw, dh, dw,
                          _p(x), _p(w), _p(b) if b is not None else None, int(relu), _p(y))
    if rc != 0:
        raise MemoryError("oracle conv2d scratch allocation failed")
    return y


def add(a, b) -> np.ndarray:
    a = _f32(a)
    b = _f32(b)
    y = np.empty_like(a)
    if a.shape == b.shape:
        lib().ora_add(a.size, _p(a), _p(b), _p(y))
    elif a.ndim == 2 and (b.ndim == 1 or (b.ndim == 2 and b.shape[0] == 1)):
        lib().ora_add_row(a.shape[0], a.shape[1], _p(a), _p(b), _p(y))
    elif a.ndim == 4 and b.ndim == 1:
        lib().ora_add_channel(a.shape[0], a.shape[1], a.shape[2] * a.shape[3], _p(a), _p(b), _p(y))
    else:
        raise ValueError("unsupported broadcast %s + %s" % (a.shape, b.shape))
    return y


def _binary(a, b, same, row, channel) -> np.ndarray:
    a = _f32(a)
    b = _f32(b)
    y = np.empty_like(a)
    if a.shape == b.shape:
        same(a.size, _p(a), _p(b), _p(y))
    elif a.ndim == 2 and (b.ndim == 1 or (b.ndim == 2 and b.shape[0] == 1)):
        row(a.shape[0], a.shape[1], _p(a), _p(b), _p(y))
    elif a.ndim == 4 and b.size == a.shape[1]:
        channel(a.shape[0], a.shape[1], a.shape[2] * a.shape[3], _p(a), _p(b), _p(y))
    else:
        raise ValueError("unsupported broadcast %s, %s" % (a.shape, b.shape))
    return y


def add_bcast(a, b) -> np.ndarray:
    """ADD with the larger operand first, any of the reference's three forms
    (a channel operand may be [C] or [C,1,1])."""
    L = lib()
    return _binary(a, b, L.ora_add, L.ora_add_row, L.ora_add_channel)


def mul(a, b) -> np.ndarray:
    """MUL with the larger operand first, in the reference's three forms."""
    L = lib()
    return _binary(a, b, L.ora_mul, L.ora_mul_row, L.ora_mul_channel)


def sigmoid(a) -> np.ndarray:
    a = _f32(a)
    y = np.empty_like(a)
    lib().ora_sigmoid(a.size, _p(a), _p(y))
    return y


def tanh(a) -> np.ndarray:
    a = _f32(a)
    y = np.empty_like(a)
    lib().ora_tanh(a.size, _p(a), _p(y))
    return y


def relu(a) -> np.ndarray:
    a = _f32(a)
    y = np.empty_like(a)
    lib().ora_relu(a.size, _p(a), _p(y))
    return y


def philox_blocks(seed: int, first: int, count: int) -> np.ndarray:
    out = np.empty((count, 4), dtype=np.uint32)
    lib().ora_philox_blocks(seed, first, count, _p(out))
    return out


def philox_normal(seed: int, first: int, count: int) -> np.ndarray:
    out = np.empty(count, dtype=np.float32)
    lib().ora_philox_normal(seed, first, count, _p(out))
    return out


# --------------------------------------------------------------------------
# whole models
# --------------------------------------------------------------------------

def _flatten_modules(model) -> List:
    import torch.nn as nn
    if isinstance(model, nn.Sequential):
        out = []
        for m in model:
            out.extend(_flatten_modules(m))
        return out
    return [model]


def run_model(model, x, variant: str = "fused_ikj", fusion: bool = True) -> np.ndarray:
    """Evaluate ``model`` on ``x`` exactly as the reference's generated runtime does.

    ``variant`` selects the reference matmul emitter; ``fused_ikj`` and
    ``loop_ikj`` give fused Linear+ReLU the bias-first order, every other
    variant and every un-fused Linear the bias-last order.  Supported modules:
    nn.Linear, nn.ReLU, nn.Conv2d (groups=1), nn.Flatten, and residual blocks
    exposing ``fc1``/``fc2`` (y = x + fc2(relu(fc1(x)))).
    """
    import torch.nn as nn

    fused_order = "bias_first" if variant in ("fused_ikj", "loop_ikj") else "bias_last"
    if type(model).__name__ == "OpMix":
        return _run_op_mix(model, _f32(x))
    h = _f32(x)
    mods = _flatten_modules(model)

    def linear(h, lin, with_relu):
        w_kn = _f32(lin.weight).T.copy()
        b = lin.bias
        if with_relu and fusion:
            return gemm(h, w_kn, b, relu=True, order=fused_order)
        y = gemm(h, w_kn, b, relu=False, order="bias_last")
        return relu(y) if with_relu else y

    i = 0
    while i < len(mods):
        m = mods[i]
        nxt = mods[i + 1] if i + 1 < len(mods) else None
        followed_by_relu = isinstance(nxt, nn.ReLU)
        if isinstance(m, nn.Linear):
            h = linear(h, m, followed_by_relu)
            i += 2 if followed_by_relu else 1
        elif isinstance(m, nn.Conv2d):
            assert m.groups == 1
            r = followed_by_relu and fusion
            h = conv2d(h, m.weight, m.bias, m.stride, m.padding, m.dilation, relu=r)
            if followed_by_relu and not fusion:
                h = relu(h)
            i += 2 if followed_by_relu else 1
        elif isinstance(m, nn.ReLU):
            h = relu(h)
            i += 1
        elif isinstance(m, nn.Flatten):
            h = h.reshape(h.shape[0], -1).copy()
            i += 1
        elif hasattr(m, "fc1") and hasattr(m, "fc2"):
            t = linear(h, m.fc1, True)
            t = linear(t, m.fc2, False)
            h = add(h, t)
            i += 1
        else:
            raise TypeError("oracle: unsupported module %r" % type(m).__name__)
    return h


def _run_op_mix(m, x: np.ndarray) -> np.ndarray:
    """forgetune_b200.workloads.OpMix in the reference's node order.  No
    MATMUL->ADD->RELU or CONV2D->RELU chain occurs, so nothing fuses
    (src/fusion.cpp:6-131): every Linear is MATMUL then a bias ADD (bias-last),
    the convolution carries its own bias (src/codegen.cpp:412-624), and ADD /
    MUL take the larger operand first (python/forgetune/export_frontend.py:16-45)."""
    def lin(h, layer):
        return gemm(h, _f32(layer.weight).T.copy(), layer.bias, relu=False, order="bias_last")

    h = conv2d(x, m.conv.weight, m.conv.bias, m.conv.stride, m.conv.padding, m.conv.dilation, relu=False)
    h = add_bcast(h, m.ch_shift)
    h = relu(mul(h, m.ch_scale))
    h = h.reshape(h.shape[0], -1).copy()
    h = lin(h, m.fc1)
    h = mul(h, m.col_scale)
    h = add_bcast(h, m.row_shift)
    a = sigmoid(h)
    b = tanh(lin(h, m.fc2))
    h = mul(a, b)
    h = add_bcast(h, a)
    return lin(h, m.head)
