"""The reference's on-disk IR (``graph.json``, schema 2.0) in and out.

Reading follows the reference's reader and its checks
(python/forgetune/graph_adapter.py:381-587, ``Graph.from_dict``; the C++
twin is src/json_io.cpp:430-790): one INPUT and one output, float32 only,
only the leading dimension may be -1, CONST data must match its shape and be
finite, operator arities, live operands, no cycles.  Deleted nodes (the
frontend keeps the untransposed weights that way) are dropped, and fused
nodes that the reference's fusion pass writes are expanded back into their
parts (FUSED_MATMUL_ADD_RELU -> MATMUL, ADD, RELU; FUSED_CONV2D_RELU ->
CONV2D, RELU; OUTPUT -> its operand), which this engine fuses again.  The
result is the IR ``compile_model`` builds from a PyTorch module, so a graph
exported by the unchanged reference frontend or CLI compiles here.

``to_graph_json`` writes the same format (src/json_io.cpp:121-200), and
``evaluate`` is a NumPy evaluation of the IR in float64 -- the correctness
gate's expected output for graphs that arrive without a PyTorch module, in
the place of the reference's ``Graph.evaluate`` (graph_adapter.py:590-).
"""

from __future__ import annotations

import json
import math
from typing import Any, Dict, List, Union

import numpy as np

from .errors import InvalidGraphError, InvalidShapeError, UnsupportedOpError
from .frontend import IRGraph

_CANONICAL = {"INPUT", "CONST", "MATMUL", "ADD", "MUL", "RELU", "SIGMOID", "TANH", "FLATTEN", "CONV2D",
              "FUSED_CONV2D_RELU", "FUSED_MATMUL_ADD_RELU", "OUTPUT"}
_ARITY = {"INPUT": (0, 0), "CONST": (0, 0), "ADD": (2, 2), "MUL": (2, 2), "MATMUL": (2, 2), "RELU": (1, 1),
          "SIGMOID": (1, 1), "TANH": (1, 1), "FLATTEN": (1, 1), "CONV2D": (2, 3), "FUSED_CONV2D_RELU": (2, 3),
          "FUSED_MATMUL_ADD_RELU": (3, 3), "OUTPUT": (1, 1)}
_CONV_KEYS = {"stride_h", "stride_w", "pad_h", "pad_w", "dilation_h", "dilation_w", "groups"}


def _is_int(v) -> bool:
    return type(v) is int


def _check_node(nd: Dict[str, Any]) -> Dict[str, Any]:
    """One node dict, checked as the reference's reader does; returns the
    normalised fields."""
    if not isinstance(nd, dict):
        raise InvalidGraphError("Node element must be a dict, got %s" % type(nd).__name__)
    nid = nd.get("id")
    if not _is_int(nid) or nid < 0:
        raise InvalidGraphError("Node id must be a non-negative int, got %r" % (nid,))
    if "name" in nd and not isinstance(nd["name"], str):
        raise InvalidGraphError("Node 'name' must be a string")
    if "deleted" in nd and type(nd["deleted"]) is not bool:
        raise InvalidGraphError("Node 'deleted' must be a boolean")
    dtype = nd.get("dtype", "f32")
    if not isinstance(dtype, str) or dtype.lower() not in ("f32", "float32"):
        raise InvalidGraphError("Unsupported node dtype: %r (only float32: 'f32' or 'float32')" % (dtype,))
    conv = nd.get("conv_attrs")
    if conv is not None:
        if not isinstance(conv, dict):
            raise InvalidGraphError("conv_attrs must be a dict")
        for k, v in conv.items():
            if k not in _CONV_KEYS:
                raise InvalidGraphError("Unknown conv_attrs key: %r" % k)
            if not _is_int(v):
                raise InvalidGraphError("conv_attrs %r must be an integer, got %r" % (k, v))
            if k in ("stride_h", "stride_w", "dilation_h", "dilation_w") and v <= 0:
                raise InvalidGraphError("conv_attrs %r must be a positive integer, got %d" % (k, v))
            if k in ("pad_h", "pad_w") and v < 0:
                raise InvalidGraphError("conv_attrs %r must be a non-negative integer, got %d" % (k, v))
            if k == "groups" and v != 1:
                raise InvalidGraphError("conv_attrs 'groups' must be 1, got %d" % v)
    op = str(nd.get("op", "")).upper()
    op = {"CONSTANT": "CONST", "FUSED_MATMUL_BIAS_RELU": "FUSED_MATMUL_ADD_RELU"}.get(op, op)
    if op not in _CANONICAL:
        raise UnsupportedOpError(op, "node %d" % nid)
    shape = nd.get("shape", [])
    if not isinstance(shape, list):
        raise InvalidShapeError("Node shape must be a list")
    for i, s in enumerate(shape):
        if not _is_int(s):
            raise InvalidShapeError("Node shape dimensions must be ints, got %r" % (s,))
        if s == -1:
            if i != 0:
                raise InvalidShapeError("Dynamic dimension -1 is only supported on the leading dimension: %s" % shape)
        elif s <= 0:
            raise InvalidShapeError("Invalid non-positive static dimension %d in shape %s" % (s, shape))
    ins = nd.get("inputs", [])
    if not isinstance(ins, list) or any(not _is_int(i) or i < 0 for i in ins):
        raise InvalidGraphError("Node inputs must be a list of non-negative ints")
    lo, hi = _ARITY[op]
    if not lo <= len(ins) <= hi:
        raise InvalidGraphError("Node op '%s' requires %d to %d inputs, got %d" % (op, lo, hi, len(ins)))
    data = nd.get("const_data", [])
    if data is None:
        if op == "CONST":
            raise InvalidGraphError("Node %d: 'const_data' cannot be null for CONST op" % nid)
        data = []
    if not isinstance(data, list):
        raise InvalidGraphError("const_data must be a list")
    for c in data:
        if type(c) is bool or not isinstance(c, (int, float)) or not math.isfinite(c) or abs(c) > 3.4028235e38:
            raise InvalidGraphError("const_data element must be a finite float32 value, got %r" % (c,))
    if op == "CONST":
        if -1 in shape:
            raise InvalidShapeError("CONST node cannot have dynamic dimension -1")
        if len(data) != int(np.prod(shape, dtype=np.int64)):
            raise InvalidShapeError("CONST node data count (%d) does not match shape %s" % (len(data), shape))
    return {"id": nid, "op": op, "inputs": list(ins), "shape": list(shape), "name": nd.get("name", ""),
            "deleted": bool(nd.get("deleted", False)), "conv": conv or {}, "data": data}


def load_graph_json(src: Union[str, bytes, Dict[str, Any]]) -> IRGraph:
    """A reference ``graph.json`` (text, bytes, a path, or the parsed dict) as
    this package's IR."""
    if isinstance(src, (bytes, bytearray)):
        src = src.decode("utf-8")
    if isinstance(src, str):
        text = src
        if not text.lstrip().startswith("{"):
            with open(text, encoding="utf-8") as f:
                text = f.read()
        try:
            d = json.loads(text)
        except json.JSONDecodeError as e:
            raise InvalidGraphError("graph JSON does not parse: %s" % e) from e
    else:
        d = src
    if not isinstance(d, dict):
        raise InvalidGraphError("Root JSON element must be an object")
    if not isinstance(d.get("nodes"), list):
        raise InvalidGraphError("Root 'nodes' property must be a list")
    major = d.get("schema_version_major", 2)
    if not _is_int(major) or major not in (1, 2):
        raise InvalidGraphError("Unsupported schema_version_major: %r (supported: 1 or 2)" % (major,))
    minor = d.get("schema_version_minor", 0)
    if not _is_int(minor) or minor != 0:
        raise InvalidGraphError("Unsupported schema_version_minor: %r (supported: 0)" % (minor,))
    max_batch = d.get("max_batch_size", 128)
    if not _is_int(max_batch) or not 1 <= max_batch <= 1_000_000:
        raise InvalidGraphError("max_batch_size must be an integer between 1 and 1000000, got %r" % (max_batch,))
    ins, outs = d.get("inputs", []), d.get("outputs", [])
    for name, ids in (("inputs", ins), ("outputs", outs)):
        if not isinstance(ids, list) or not ids:
            raise InvalidGraphError("Graph has empty %s list" % name)
        if len(ids) > 1:
            raise InvalidGraphError("ForgeTune supports single-input, single-output graphs, got %d %s"
                                    % (len(ids), name))
        if any(not _is_int(i) or i < 0 for i in ids):
            raise InvalidGraphError("%s must be non-negative node ids" % name)

    nodes: Dict[int, Dict[str, Any]] = {}
    for nd in d["nodes"]:
        n = _check_node(nd)
        if n["id"] in nodes:
            raise InvalidGraphError("Duplicate node ID in JSON: %d" % n["id"])
        nodes[n["id"]] = n
    live = {i: n for i, n in nodes.items() if not n["deleted"]}
    in_id, out_id = ins[0], outs[0]
    if in_id not in nodes or nodes[in_id]["deleted"] or nodes[in_id]["op"] != "INPUT":
        raise InvalidGraphError("Graph input node %d must be a live INPUT node" % in_id)
    if {i for i, n in live.items() if n["op"] == "INPUT"} != {in_id}:
        raise InvalidGraphError("live INPUT nodes must be exactly the declared input")
    if out_id not in nodes or nodes[out_id]["deleted"]:
        raise InvalidGraphError("Graph output node %d does not exist or is deleted" % out_id)
    for i, n in live.items():
        for o in n["inputs"]:
            if o not in nodes:
                raise InvalidGraphError("Node %d references missing operand node %d" % (i, o))
            if nodes[o]["deleted"]:
                raise InvalidGraphError("Node %d references deleted operand node %d" % (i, o))

    # topological order of the live nodes (depth-first, inputs first)
    order: List[int] = []
    state: Dict[int, int] = {}
    for root in sorted(live):
        stack = [(root, 0)]
        while stack:
            nid, k = stack.pop()
            if k == 0:
                if state.get(nid) == 2:
                    continue
                if state.get(nid) == 1:
                    raise InvalidGraphError("graph has a cycle through node %d" % nid)
                state[nid] = 1
            ins_n = live[nid]["inputs"]
            if k < len(ins_n):
                stack.append((nid, k + 1))
                if state.get(ins_n[k]) != 2:
                    if state.get(ins_n[k]) == 1:
                        raise InvalidGraphError("graph has a cycle through node %d" % ins_n[k])
                    stack.append((ins_n[k], 0))
            else:
                state[nid] = 2
                order.append(nid)

    in_shape = live[in_id]["shape"]
    g = IRGraph(max_batch_size=max_batch, dynamic=bool(in_shape) and in_shape[0] == -1)
    env: Dict[int, int] = {}
    for nid in order:
        n = live[nid]
        op, shape, name = n["op"], n["shape"], n["name"]
        a = [env[i] for i in n["inputs"]]
        if op == "INPUT":
            env[nid] = g.add("INPUT", [], shape, name)
            g.input_id = env[nid]
        elif op == "CONST":
            env[nid] = g.add("CONST", [], shape, name, const=np.asarray(n["data"], np.float32).reshape(shape))
        elif op == "OUTPUT":
            env[nid] = a[0]
        elif op == "FUSED_MATMUL_ADD_RELU":
            mm = g.add("MATMUL", a[:2], shape, name + "_mm")
            ad = g.add("ADD", [mm, a[2]], shape, name + "_bias")
            env[nid] = g.add("RELU", [ad], shape, name)
        elif op in ("CONV2D", "FUSED_CONV2D_RELU"):
            c = n["conv"]
            conv = dict(sh=c.get("stride_h", 1), sw=c.get("stride_w", 1), ph=c.get("pad_h", 0),
                        pw=c.get("pad_w", 0), dh=c.get("dilation_h", 1), dw=c.get("dilation_w", 1))
            cv = g.add("CONV2D", a, shape, name if op == "CONV2D" else name + "_conv", conv=conv)
            env[nid] = cv if op == "CONV2D" else g.add("RELU", [cv], shape, name)
        else:
            env[nid] = g.add(op, a, shape, name)
    g.output_id = env[out_id]
    return g


def to_graph_json(g: IRGraph, indent: int = 2) -> str:
    """The IR in the reference's schema 2.0 (src/json_io.cpp:121-200)."""
    nodes = []
    for n in g.nodes:
        nd: Dict[str, Any] = {"id": n.id, "op": n.op, "name": n.name, "inputs": list(n.inputs),
                              "shape": list(n.shape), "dtype": "f32",
                              "const_data": [float(v) for v in np.asarray(n.const, np.float32).ravel()]
                              if n.const is not None else [], "deleted": False}
        if n.op == "CONV2D":
            c = n.conv or {}
            nd["conv_attrs"] = {"stride_h": c.get("sh", 1), "stride_w": c.get("sw", 1), "pad_h": c.get("ph", 0),
                                "pad_w": c.get("pw", 0), "dilation_h": c.get("dh", 1),
                                "dilation_w": c.get("dw", 1), "groups": 1}
        nodes.append(nd)
    return json.dumps({"schema_version_major": 2, "schema_version_minor": 0, "max_batch_size": g.max_batch_size,
                       "inputs": [g.input_id], "outputs": [g.output_id], "nodes": nodes}, indent=indent)


def _conv2d(x: np.ndarray, w: np.ndarray, b, c: Dict[str, int]) -> np.ndarray:
    B, C, H, W = x.shape
    O, _, KH, KW = w.shape
    sh, sw, ph, pw, dh, dw = c.get("sh", 1), c.get("sw", 1), c.get("ph", 0), c.get("pw", 0), c.get("dh", 1), \
        c.get("dw", 1)
    Ho = (H + 2 * ph - dh * (KH - 1) - 1) // sh + 1
    Wo = (W + 2 * pw - dw * (KW - 1) - 1) // sw + 1
    xp = np.zeros((B, C, H + 2 * ph, W + 2 * pw), x.dtype)
    xp[:, :, ph:ph + H, pw:pw + W] = x
    cols = np.empty((B, C, KH, KW, Ho, Wo), x.dtype)
    for i in range(KH):
        for j in range(KW):
            cols[:, :, i, j] = xp[:, :, i * dh:i * dh + sh * (Ho - 1) + 1:sh, j * dw:j * dw + sw * (Wo - 1) + 1:sw]
    y = np.einsum("bckhij,ockh->boij", cols.reshape(B, C, KH, KW, Ho, Wo), w, optimize=True)
    if b is not None:
        y = y + b.reshape(1, O, 1, 1)
    return y


def evaluate(g: IRGraph, x: np.ndarray) -> np.ndarray:
    """The IR on a batch, in float64 (NaN-keeping ReLU as in the reference);
    returns float32."""
    vals: Dict[int, np.ndarray] = {}
    for n in g.nodes:
        a = [vals[i] for i in n.inputs]
        if n.op == "INPUT":
            v = np.asarray(x, np.float64)
        elif n.op == "CONST":
            v = np.asarray(n.const, np.float64)
        elif n.op == "MATMUL":
            v = a[0] @ a[1]
        elif n.op == "ADD":
            v = a[0] + a[1]
        elif n.op == "MUL":
            v = a[0] * a[1]
        elif n.op == "RELU":
            v = np.where(np.isnan(a[0]) | (a[0] > 0), a[0], 0.0)
        elif n.op == "SIGMOID":
            v = 1.0 / (1.0 + np.exp(-a[0]))
        elif n.op == "TANH":
            v = np.tanh(a[0])
        elif n.op == "FLATTEN":
            v = a[0].reshape(a[0].shape[0], -1)
        elif n.op == "CONV2D":
            v = _conv2d(a[0], a[1], a[2] if len(a) > 2 else None, n.conv or {})
        elif n.op == "OUTPUT":
            v = a[0]
        else:
            raise UnsupportedOpError(n.op)
        vals[n.id] = v
    return vals[g.output_id].astype(np.float32)
