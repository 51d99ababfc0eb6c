"""Lower a ``torch.nn.Module`` to the reference IR.

``torch.export`` traces the module (with a symbolic leading batch dimension
when ``dynamic_batch``) and every ATen call is lowered to the reference's IR
vocabulary, with the reference's conventions
(python/forgetune/export_frontend.py):

* ``aten.linear(x, W, b)`` -> CONST W^T [K, N], MATMUL(x, W^T), ADD(mm, b)  (:224-297)
* ``aten.conv2d`` / ``aten.convolution`` (groups 1, not transposed) -> CONV2D (:622-698)
* ``aten.add`` / ``aten.mul`` -> ADD / MUL with the larger operand first (:18-46, :386-417)
* ``aten.relu`` / ``sigmoid`` / ``tanh`` -> RELU / SIGMOID / TANH
* ``aten.flatten(x, 1, -1)`` and ``view``/``reshape`` to [B, -1] -> FLATTEN (:486-620)

Only one float32 input and one output are supported, as in the reference;
only the leading dimension may be dynamic.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence

import numpy as np
import torch

from .errors import InvalidGraphError, InvalidShapeError, UnsupportedOpError

# op codes shared with the native engine (csrc/engine.hpp: OpKind)
OPS = {
    "INPUT": 0, "CONST": 1, "MATMUL": 2, "ADD": 3, "RELU": 4, "OUTPUT": 5,
    "MUL": 7, "SIGMOID": 8, "TANH": 9, "CONV2D": 10, "FLATTEN": 11,
}


@dataclass
class IRNode:
    id: int
    op: str
    inputs: List[int]
    shape: List[int]
    name: str = ""
    const: Optional[np.ndarray] = None
    conv: Optional[Dict[str, int]] = None


@dataclass
class IRGraph:
    nodes: List[IRNode] = field(default_factory=list)
    input_id: int = -1
    output_id: int = -1
    max_batch_size: int = 128
    dynamic: bool = False

    def add(self, op: str, inputs: Sequence[int], shape: Sequence[int], name: str = "",
            const: Optional[np.ndarray] = None, conv: Optional[Dict[str, int]] = None) -> int:
        nid = len(self.nodes)
        self.nodes.append(IRNode(nid, op, list(inputs), [int(d) for d in shape], name, const, conv))
        return nid

    def shape(self, nid: int) -> List[int]:
        return self.nodes[nid].shape


def _broadcast_order(g: IRGraph, a: int, b: int):
    """Larger operand first and the broadcast result shape (export_frontend.py:18-46)."""
    sa, sb = g.shape(a), g.shape(b)
    r = max(len(sa), len(sb))
    pa = [1] * (r - len(sa)) + list(sa)
    pb = [1] * (r - len(sb)) + list(sb)
    out = []
    for da, db in zip(pa, pb):
        if da == -1 or db == -1:
            out.append(-1)
        elif da == 1:
            out.append(db)
        elif db == 1 or da == db:
            out.append(da)
        else:
            raise InvalidShapeError("cannot broadcast shapes %s and %s" % (sa, sb))

    def weight(s):
        w = 1
        for d in s:
            w *= 1000 if d == -1 else (d if d > 1 else 1)
        return w

    if len(sa) < len(sb) or (len(sa) == len(sb) and weight(sa) < weight(sb)):
        return [b, a], out
    return [a, b], out


def _shape_of(node) -> List[int]:
    val = node.meta.get("val")
    if val is None:
        raise InvalidGraphError("node %s has no shape metadata" % node.name)
    dims = []
    for i, d in enumerate(val.shape):
        if isinstance(d, int):
            dims.append(int(d))
        else:
            if i != 0:
                raise InvalidShapeError("only the leading (batch) dimension may be dynamic, got %s" % list(val.shape))
            dims.append(-1)
    return dims


def _pair(v, default):
    if v is None:
        return (default, default)
    if isinstance(v, (list, tuple)):
        return (int(v[0]), int(v[1] if len(v) > 1 else v[0]))
    return (int(v), int(v))


def export_to_ir(model: torch.nn.Module, example_inputs, dynamic_batch: bool = False,
                 max_batch_size: int = 128) -> IRGraph:
    """torch.export ``model`` and lower it to an :class:`IRGraph`."""
    if len(example_inputs) != 1:
        raise ValueError("exactly one example input is supported, got %d" % len(example_inputs))
    x = example_inputs[0]
    if not isinstance(x, torch.Tensor) or x.dtype != torch.float32:
        raise TypeError("example input must be a float32 torch.Tensor")
    for name, p in model.named_parameters():
        if p.dtype != torch.float32:
            raise TypeError("parameter '%s' has dtype %s; only float32 models are supported" % (name, p.dtype))
    dyn = None
    if dynamic_batch:
        if x.shape[0] > max_batch_size:
            raise InvalidShapeError("example batch %d exceeds max_batch_size=%d" % (x.shape[0], max_batch_size))
        dyn = ({0: torch.export.Dim("batch", min=1, max=max_batch_size)},)
    try:
        ep = torch.export.export(model, (x,), dynamic_shapes=dyn)
    except Exception as e:  # torch raises many types here
        raise InvalidGraphError("torch.export failed: %s" % e) from e

    sig = ep.graph_signature
    params = {}
    for spec in sig.input_specs:
        if spec.target is not None:
            params[spec.arg.name] = spec.target
    state = ep.state_dict
    consts = getattr(ep, "constants", {}) or {}

    g = IRGraph(max_batch_size=max_batch_size, dynamic=dynamic_batch)
    env: Dict[str, int] = {}

    def const_node(name: str, arr: np.ndarray) -> int:
        arr = np.ascontiguousarray(arr, dtype=np.float32)
        if not np.all(np.isfinite(arr)):
            raise InvalidGraphError("constant %s holds NaN or Inf" % name)
        return g.add("CONST", [], list(arr.shape), name, const=arr)

    for node in ep.graph_module.graph.nodes:
        if node.op == "placeholder":
            if node.name in params:
                t = params[node.name]
                tensor = state[t] if t in state else consts[t]
                env[node.name] = const_node(node.name, tensor.detach().cpu().numpy())
            else:
                if g.input_id >= 0:
                    raise ValueError("only single-input models are supported")
                shape = _shape_of(node)
                g.input_id = env[node.name] = g.add("INPUT", [], shape, node.name)
            continue
        if node.op == "output":
            outs = node.args[0]
            if not isinstance(outs, (list, tuple)) or len(outs) != 1:
                raise ValueError("only single-output models are supported")
            g.output_id = env[outs[0].name]
            continue
        if node.op != "call_function":
            raise UnsupportedOpError(str(node.op), node.name)
        target = str(node.target)
        args = node.args
        if "aten.linear" in target:
            xi = env[args[0].name]
            wi = env[args[1].name]
            w = g.nodes[wi].const
            if w is None or w.ndim != 2:
                raise UnsupportedOpError("aten.linear", "weight must be a 2-D parameter")
            if len(g.shape(xi)) != 2:
                raise UnsupportedOpError("aten.linear", "input must be rank 2 [B, K]; flatten first")
            N, K = w.shape
            wt = const_node(args[1].name + "_transposed", w.T.copy())
            mm = g.add("MATMUL", [xi, wt], [g.shape(xi)[0], N], node.name + "_matmul")
            if len(args) > 2 and args[2] is not None:
                env[node.name] = g.add("ADD", [mm, env[args[2].name]], [g.shape(xi)[0], N], node.name)
            else:
                env[node.name] = mm
        elif "aten.relu" in target or "aten.sigmoid" in target or "aten.tanh" in target:
            op = "RELU" if "relu" in target else ("SIGMOID" if "sigmoid" in target else "TANH")
            xi = env[args[0].name]
            env[node.name] = g.add(op, [xi], g.shape(xi), node.name)
        elif "aten.add" in target or "aten.mul" in target:
            op = "ADD" if "aten.add" in target else "MUL"
            a, b = args[0], args[1]
            if not hasattr(a, "name") or not hasattr(b, "name"):
                raise UnsupportedOpError(target, "scalar operands are not supported")
            alpha = node.kwargs.get("alpha", 1) if node.kwargs else 1
            if alpha != 1:
                raise UnsupportedOpError(target, "alpha != 1")
            ins, out = _broadcast_order(g, env[a.name], env[b.name])
            env[node.name] = g.add(op, ins, out, node.name)
        elif "conv2d" in target or "aten.convolution" in target:
            xi = env[args[0].name]
            wi = env[args[1].name]
            bi = env[args[2].name] if len(args) > 2 and args[2] is not None else None
            if "aten.convolution" in target:
                stride, padding, dilation = args[3], args[4], args[5]
                if args[6]:
                    raise UnsupportedOpError(target, "transposed convolution")
                groups = args[8]
            else:
                stride = args[3] if len(args) > 3 else 1
                padding = args[4] if len(args) > 4 else 0
                dilation = args[5] if len(args) > 5 else 1
                groups = args[6] if len(args) > 6 else 1
            if groups != 1:
                raise UnsupportedOpError(target, "groups=%s (only 1 is supported)" % groups)
            if isinstance(padding, str):
                raise UnsupportedOpError(target, "string padding '%s'" % padding)
            sh, sw = _pair(stride, 1)
            ph, pw = _pair(padding, 0)
            dh, dw = _pair(dilation, 1)
            xs, ws = g.shape(xi), g.shape(wi)
            if len(xs) != 4 or len(ws) != 4 or xs[1] != ws[1]:
                raise InvalidShapeError("CONV2D needs NCHW input and matching OIHW weight, got %s, %s" % (xs, ws))
            Ho = (xs[2] + 2 * ph - (dh * (ws[2] - 1) + 1)) // sh + 1
            Wo = (xs[3] + 2 * pw - (dw * (ws[3] - 1) + 1)) // sw + 1
            if Ho <= 0 or Wo <= 0:
                raise InvalidShapeError("CONV2D output would be empty")
            ins = [xi, wi] + ([bi] if bi is not None else [])
            env[node.name] = g.add("CONV2D", ins, [xs[0], ws[0], Ho, Wo], node.name,
                                   conv=dict(sh=sh, sw=sw, ph=ph, pw=pw, dh=dh, dw=dw))
        elif "aten.flatten" in target or "aten.view" in target or "aten.reshape" in target \
                or "aten._unsafe_view" in target:
            xi = env[args[0].name]
            xs = g.shape(xi)
            out = _shape_of(node)
            if len(out) != 2 or len(xs) not in (2, 4) or (xs[0] != out[0]):
                raise UnsupportedOpError(target, "only flattening [B, ...] to [B, features] is supported")
            if xs == out:
                env[node.name] = xi
            else:
                env[node.name] = g.add("FLATTEN", [xi], out, node.name)
        elif "aten.dropout" in target or "aten.clone" in target or "aten.contiguous" in target \
                or "aten.alias" in target or "aten.detach" in target:
            env[node.name] = env[args[0].name]
        elif "aten.sym_size" in target:
            continue
        else:
            raise UnsupportedOpError(target, node.name)
    if g.input_id < 0 or g.output_id < 0:
        raise InvalidGraphError("graph has no input or no output")
    return g
