"""Writes tests/golden/graph_json/: small models exported to graph.json by the
reference's own frontend (python/forgetune/export_frontend.py,
export_to_forgetune_ir + Graph.to_json), with a seeded input and the PyTorch
output for each.  Run in a checkout that has the reference next to it:

    python tests/golden/make_graph_json.py /path/to/reference

``mlp_fused.json`` is ``mlp.json`` rewritten the way the reference's C++
fusion pass leaves a graph (src/fusion.cpp:53-120: a FUSED_MATMUL_ADD_RELU
node with inputs {x, W, bias} in place of the RELU, the MATMUL / ADD / RELU
marked deleted) plus an OUTPUT node, so the reader's handling of fused and
deleted nodes is tested on that shape of file.
"""

import json
import os
import sys

import numpy as np
import torch
import torch.nn as nn

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "graph_json")


class Residual(nn.Module):
    def __init__(self):
        super().__init__()
        self.a = nn.Linear(4, 4)
        self.b = nn.Linear(4, 4)

    def forward(self, x):
        return x + self.b(torch.relu(self.a(x)))


def models():
    torch.manual_seed(0)
    yield "mlp", nn.Sequential(nn.Linear(6, 5), nn.ReLU(), nn.Linear(5, 3)), (6,), True, 64
    torch.manual_seed(1)
    yield "cnn", nn.Sequential(nn.Conv2d(2, 3, 3, stride=2, padding=1), nn.ReLU(), nn.Flatten(),
                               nn.Linear(48, 2)), (2, 8, 8), True, 64
    torch.manual_seed(2)
    yield "residual", Residual(), (4,), True, 64
    torch.manual_seed(3)
    yield "activations_static", nn.Sequential(nn.Linear(4, 4), nn.Sigmoid(), nn.Tanh()), (4,), False, 3


def fused_variant(d):
    """mlp.json as the reference's fusion pass would leave it."""
    d = json.loads(json.dumps(d))
    nodes = {n["id"]: n for n in d["nodes"]}
    next_id = max(nodes) + 1
    for relu in [n for n in d["nodes"] if n["op"] == "RELU" and not n["deleted"]]:
        add = nodes[relu["inputs"][0]]
        if add["op"] != "ADD":
            continue
        mm_id = add["inputs"][0] if nodes[add["inputs"][0]]["op"] == "MATMUL" else add["inputs"][1]
        bias_id = add["inputs"][1] if mm_id == add["inputs"][0] else add["inputs"][0]
        mm = nodes[mm_id]
        for n in (mm, add):
            n["deleted"] = True
        relu["op"] = "FUSED_MATMUL_ADD_RELU"
        relu["inputs"] = [mm["inputs"][0], mm["inputs"][1], bias_id]
    out = {"id": next_id, "op": "OUTPUT", "name": "output", "inputs": [d["outputs"][0]],
           "shape": nodes[d["outputs"][0]]["shape"], "dtype": "f32", "const_data": [], "deleted": False}
    d["nodes"].append(out)
    d["outputs"] = [next_id]
    return d


def main(ref_root):
    sys.path.insert(0, os.path.join(ref_root, "python"))
    from forgetune.export_frontend import export_to_forgetune_ir
    os.makedirs(OUT, exist_ok=True)
    for name, m, shape, dynamic, max_batch in models():
        m.eval()
        batch = 5 if dynamic else max_batch
        example = torch.randn((2 if dynamic else batch,) + shape)
        g = export_to_forgetune_ir(m, (example,), dynamic_batch=dynamic, max_batch_size=max_batch)
        d = json.loads(g.to_json())
        x = np.random.default_rng(7).standard_normal((batch,) + shape).astype(np.float32)
        with torch.no_grad():
            y = m(torch.from_numpy(x)).numpy()
        with open(os.path.join(OUT, name + ".json"), "w") as f:
            json.dump(d, f, indent=1)
        np.savez(os.path.join(OUT, name + ".npz"), x=x, y=y)
        if name == "mlp":
            with open(os.path.join(OUT, "mlp_fused.json"), "w") as f:
                json.dump(fused_variant(d), f, indent=1)
        print(name, len(d["nodes"]), "nodes")


if __name__ == "__main__":
    sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
    from oracle.build_ref import reference_root
    main(sys.argv[1] if len(sys.argv) > 1 else reference_root())
