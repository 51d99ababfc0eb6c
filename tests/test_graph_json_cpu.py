"""The reference's graph.json on CPU: fixtures exported by the reference's
own frontend (tests/golden/make_graph_json.py) load into the same IR and
launch list as the same model lowered by this package, evaluate to the
PyTorch outputs, survive a write / read round trip, and malformed files are
rejected with the reference reader's checks."""

import copy
import json
import os

import numpy as np
import pytest
import torch
import torch.nn as nn

from forgetune_b200 import InvalidGraphError, InvalidShapeError, UnsupportedOpError, _native
from forgetune_b200 import compile_graph_json, export_to_ir, load_graph_json, to_graph_json
from forgetune_b200.graph_blob import _live_nodes, serialize
from forgetune_b200.ir_json import evaluate

GJ = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "graph_json")
NAMES = ["mlp", "cnn", "residual", "activations_static"]


def fixture(name):
    with open(os.path.join(GJ, name + ".json")) as f:
        d = json.load(f)
    return d, np.load(os.path.join(GJ, (name if name != "mlp_fused" else "mlp") + ".npz"))


@pytest.mark.parametrize("name", NAMES + ["mlp_fused"])
def test_fixture_loads_and_evaluates_to_the_pytorch_output(name):
    d, io = fixture(name)
    ir = load_graph_json(d)
    assert ir.dynamic == (name != "activations_static")
    assert np.allclose(evaluate(ir, io["x"]), io["y"], atol=1e-5, rtol=1e-5)
    again = load_graph_json(to_graph_json(ir))
    assert np.array_equal(evaluate(again, io["x"]), evaluate(ir, io["x"]))
    assert [n.op for n in again.nodes] == [n.op for n in ir.nodes]


def rebuilt(name):
    """The fixture's model, rebuilt with the generator's seed."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("mk", os.path.join(os.path.dirname(GJ), "make_graph_json.py"))
    mk = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mk)
    for n, m, shape, dynamic, max_batch in mk.models():
        if n == name:
            return m.eval(), shape, dynamic, max_batch
    raise KeyError(name)


@pytest.mark.parametrize("name", NAMES)
def test_same_launch_list_as_the_module_lowered_here(name):
    m, shape, dynamic, max_batch = rebuilt(name)
    ex = torch.randn((2 if dynamic else max_batch,) + shape)
    mine = export_to_ir(m, (ex,), dynamic_batch=dynamic, max_batch_size=max_batch)
    theirs = load_graph_json(fixture(name)[0])
    for fusion in (False, True):
        a = _native.describe_blob(serialize(mine, enable_fusion=fusion, bias_first_fused=True))
        b = _native.describe_blob(serialize(theirs, enable_fusion=fusion, bias_first_fused=True))
        key = lambda d: [(s["kind"], s["K"], s["N"], s["epi"]) for s in d["steps"]]
        assert key(a) == key(b)
        assert a["arena_bytes"] == b["arena_bytes"]
    # the weights that reach the output are the same floats
    wm = [mine.nodes[i].const for i in _live_nodes(mine) if mine.nodes[i].op == "CONST"]
    wt = [theirs.nodes[i].const for i in _live_nodes(theirs) if theirs.nodes[i].op == "CONST"]
    assert sorted(w.tobytes() for w in wm) == sorted(w.tobytes() for w in wt)


def mutate(d, fn):
    d = copy.deepcopy(d)
    fn(d)
    return d


def node(d, op, live=True):
    return next(n for n in d["nodes"] if n["op"] == op and n["deleted"] != live)


BAD = {
    "no nodes": (lambda d: d.pop("nodes"), InvalidGraphError),
    "schema 3": (lambda d: d.update(schema_version_major=3), InvalidGraphError),
    "minor 1": (lambda d: d.update(schema_version_minor=1), InvalidGraphError),
    "two inputs": (lambda d: d.update(inputs=[d["inputs"][0], d["inputs"][0] + 100]), InvalidGraphError),
    "no outputs": (lambda d: d.update(outputs=[]), InvalidGraphError),
    "max batch 0": (lambda d: d.update(max_batch_size=0), InvalidGraphError),
    "f64": (lambda d: node(d, "MATMUL").update(dtype="f64"), InvalidGraphError),
    "dyn dim 1": (lambda d: node(d, "INPUT").update(shape=[2, -1]), InvalidShapeError),
    "zero dim": (lambda d: node(d, "RELU").update(shape=[-1, 0]), InvalidShapeError),
    "const count": (lambda d: node(d, "CONST").update(const_data=[1.0]), InvalidShapeError),
    "const inf": (lambda d: node(d, "CONST").update(const_data=[float("inf")] * len(node(d, "CONST")["const_data"])),
                  InvalidGraphError),
    "unknown op": (lambda d: node(d, "RELU").update(op="GELU"), UnsupportedOpError),
    "arity": (lambda d: node(d, "RELU").update(inputs=[]), InvalidGraphError),
    "deleted operand": (lambda d: node(d, "RELU").update(inputs=[node(d, "CONST", live=False)["id"]]),
                        InvalidGraphError),
    "missing operand": (lambda d: node(d, "RELU").update(inputs=[999]), InvalidGraphError),
    "duplicate id": (lambda d: d["nodes"].append(dict(node(d, "RELU"))), InvalidGraphError),
    "cycle": (lambda d: node(d, "MATMUL").update(inputs=[node(d, "RELU")["id"], node(d, "MATMUL")["inputs"][1]]),
              InvalidGraphError),
    "input not INPUT": (lambda d: d.update(inputs=[node(d, "RELU")["id"]]), InvalidGraphError),
    "deleted output": (lambda d: d.update(outputs=[node(d, "CONST", live=False)["id"]]), InvalidGraphError),
}


@pytest.mark.parametrize("case", sorted(BAD))
def test_malformed_graphs_are_rejected(case):
    fn, err = BAD[case]
    d = mutate(fixture("mlp")[0], fn)
    with pytest.raises(err):
        load_graph_json(d)


def test_bad_conv_attrs_are_rejected():
    d = fixture("cnn")[0]
    for attrs in ({"groups": 2}, {"stride_h": 0}, {"pad_w": -1}, {"bogus": 1}, {"stride_w": 1.5}):
        bad = copy.deepcopy(d)
        node(bad, "CONV2D")["conv_attrs"].update(attrs)
        with pytest.raises(InvalidGraphError):
            load_graph_json(bad)


def test_text_bytes_and_path_sources(tmp_path):
    d = fixture("mlp")[0]
    p = tmp_path / "graph.json"
    p.write_text(json.dumps(d))
    a = [n.op for n in load_graph_json(str(p)).nodes]
    assert a == [n.op for n in load_graph_json(json.dumps(d)).nodes] == [n.op for n in
                                                                         load_graph_json(json.dumps(d).encode()).nodes]
    with pytest.raises(InvalidGraphError):
        load_graph_json("{not json")


def test_compile_graph_json_without_a_gpu_builds_the_artifact(tmp_path):
    if _native.device_count() > 0:
        pytest.skip("covered by the GPU test")
    cm = compile_graph_json(os.path.join(GJ, "cnn.json"), output_dir=str(tmp_path), autotune=True,
                            enable_fusion=True)
    man = cm.manifest()
    assert os.path.isfile(man["artifacts"]["shared_library"])
    assert man["optimization_summary"]["autotune"]["status"] == "skipped"
    assert man["optimization_summary"]["verification"]["status"] == "skipped"
    assert man["input_shape"] == [-1, 2, 8, 8] and man["output_shape"] == [-1, 2]
    cm.close()
