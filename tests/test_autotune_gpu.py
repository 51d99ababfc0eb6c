"""The on-device autotuner: every candidate through the correctness gate,
interleaved timing, per-step and per-batch-range selection by the
reference's rules, the table carried in the graph blob, the cache, and
compile_model(autotune=True) end to end."""

import os

import numpy as np
import pytest
import torch
import torch.nn as nn

from forgetune_b200 import _native, compile_model, workloads
from forgetune_b200.autotuner import Autotuner
from forgetune_b200.frontend import export_to_ir
from forgetune_b200.graph_blob import serialize, tuning_of, with_tuning

pytestmark = pytest.mark.gpu


def torch_oracle(m):
    def run(x):
        with torch.no_grad():
            return m(torch.from_numpy(np.ascontiguousarray(x))).numpy()
    return run


def test_tune_tiny_mlp_selects_by_the_rules(tmp_path):
    m = workloads.tiny_mlp().eval()
    ir = export_to_ir(m, (torch.randn(2, 784),), True, 65536)
    blob = serialize(ir, enable_fusion=True, bias_first_fused=True)
    ex = workloads.seeded_input((64, 784)).numpy()
    tuner = Autotuner(cache_dir=str(tmp_path / "cache"), device=torch.cuda.current_device())
    table, rep = tuner.tune(blob, torch_oracle(m), ex, (-1, 784), str(tmp_path / "art"),
                            tuning_batch_sizes=[16, 512, 65536])
    evs = rep["candidate_evaluations"]
    assert len(evs) == 8 and evs[0]["candidate"]["candidate_id"] == "engine_default"
    assert evs[0]["status"] == "passed"
    passed = {e["candidate"]["candidate_id"]: e for e in evs if e["status"] == "passed"}
    assert len(passed) >= 2
    for e in passed.values():
        assert set(e["per_batch_step_ms"]) == {"16", "512", "65536"}
    # every non-baseline choice is at least 5 % faster than the baseline on its steps
    for sel in rep["selections"]:
        if sel["selected"] == "engine_default" or sel["batch"] in rep["safeguard_reverted_batches"]:
            continue
        b, steps = str(sel["batch"]), sel["steps"]
        cost = {cid: sum(e["per_batch_step_ms"][b][s] for s in steps) for cid, e in passed.items()}
        assert cost[sel["selected"]] * 1.05 <= cost["engine_default"] + 1e-4, sel
    assert os.path.isfile(tmp_path / "art" / "autotuning_report.json")

    # the tuned blob runs and matches the model at batches inside every range
    eng = _native.EngineModel(with_tuning(blob, table))
    eng.set_devices([torch.cuda.current_device()])
    rng = np.random.default_rng(5)
    for b in (1, 16, 100, 512, 3000, 20000):
        x = rng.standard_normal((b, 784)).astype(np.float32)
        y = np.zeros((b, 10), np.float32)
        assert eng.run(x, y) == 0, _native.last_error()
        assert np.allclose(y, torch_oracle(m)(x), atol=1e-4, rtol=1e-4), b
    eng.close()

    # the cache returns the same table without timing again
    table2, rep2 = tuner.tune(blob, torch_oracle(m), ex, (-1, 784), str(tmp_path / "art2"),
                              tuning_batch_sizes=[16, 512, 65536])
    assert rep2["cache_hit"] is True and table2 == table


def test_compile_model_autotune_end_to_end(tmp_path, monkeypatch):
    monkeypatch.chdir(tmp_path)  # the default tuning cache lives under ./build
    torch.manual_seed(0)
    m = nn.Sequential(nn.Linear(256, 512), nn.ReLU(), nn.Linear(512, 10)).eval()
    cm = compile_model(m, (torch.randn(8, 256),), output_dir=str(tmp_path / "out"), autotune=True,
                       enable_fusion=True, dynamic_batch=True, max_batch_size=8192,
                       tuning_batch_sizes=[8, 1024, 8192])
    summary = cm.manifest()["optimization_summary"]["autotune"]
    assert summary["status"] == "tuned", summary
    with open(cm.manifest()["artifacts"]["graph_blob"], "rb") as f:
        assert tuning_of(f.read()) == summary["table"]
    assert os.path.isfile(summary["report"])
    assert os.path.isdir(tmp_path / "build" / "tuning_cache")
    x = np.random.default_rng(1).standard_normal((3000, 256)).astype(np.float32)
    got = cm.run(x)
    assert np.allclose(got, torch_oracle(m)(x), atol=1e-4, rtol=1e-4)
    assert np.array_equal(got.view(np.uint32), cm.run(x).view(np.uint32))
    cm.close()
