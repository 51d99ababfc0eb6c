"""compile_graph_json on the GPU: graphs written by the reference's frontend
run through the same engine as compile_model and give the PyTorch outputs;
a full-size graph written to graph.json gives the same bits as the module
compiled directly."""

import json
import os

import numpy as np
import pytest
import torch

from forgetune_b200 import compile_graph_json, compile_model, export_to_ir, to_graph_json, workloads

pytestmark = pytest.mark.gpu

GJ = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "graph_json")


@pytest.mark.parametrize("name,io", [("mlp", "mlp"), ("mlp_fused", "mlp"), ("cnn", "cnn"), ("residual", "residual"),
                                     ("activations_static", "activations_static")])
@pytest.mark.parametrize("policy", ["auto", "simt_exact", "tcgen05"])
def test_reference_graph_json_runs(name, io, policy, tmp_path):
    data = np.load(os.path.join(GJ, io + ".npz"))
    cm = compile_graph_json(os.path.join(GJ, name + ".json"), output_dir=str(tmp_path), autotune=False,
                            enable_fusion=True, kernel_variant="fused_ikj", gpu_kernel=policy)
    assert cm.manifest()["optimization_summary"]["verification"]["status"] == "passed"
    got = cm.run(data["x"])
    assert np.allclose(got, data["y"], atol=1e-4, rtol=1e-4), float(np.max(np.abs(got - data["y"])))
    cm.close()


def test_full_size_graph_json_matches_the_module_bitwise(tmp_path):
    m = workloads.tiny_mlp().eval()
    ex = workloads.seeded_input((4, 784))
    ir = export_to_ir(m, (ex,), dynamic_batch=True, max_batch_size=8192)
    path = tmp_path / "graph.json"
    path.write_text(to_graph_json(ir))
    x = np.random.default_rng(3).standard_normal((4096, 784)).astype(np.float32)
    outs = []
    for build in ("json", "module"):
        kw = dict(output_dir=str(tmp_path / build), autotune=False, enable_fusion=True, kernel_variant="fused_ikj",
                  gpu_kernel="auto", verify=False, max_workspace_bytes=4 << 30)
        if build == "json":
            cm = compile_graph_json(str(path), example_input=ex.numpy(), **kw)
        else:
            cm = compile_model(m, (ex,), dynamic_batch=True, max_batch_size=8192, **kw)
        outs.append(cm.run(x))
        cm.close()
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))


def test_graph_json_with_the_autotuner(tmp_path, monkeypatch):
    monkeypatch.chdir(tmp_path)
    data = np.load(os.path.join(GJ, "cnn.npz"))
    cm = compile_graph_json(os.path.join(GJ, "cnn.json"), output_dir=str(tmp_path / "out"), autotune=True,
                            enable_fusion=True)
    assert cm.manifest()["optimization_summary"]["autotune"]["status"] == "tuned"
    assert np.allclose(cm.run(data["x"]), data["y"], atol=1e-4, rtol=1e-4)
    cm.close()
