"""The autotuner's host logic, no GPU: candidate-space contract (the
reference's get_candidate_space rules), selection rules (>= 5 % over the
baseline, 5 % tie band broken by simplicity), batch ranges, the tuning table
in the graph blob and the engine's validation of it."""

import ctypes

import pytest
import torch

from forgetune_b200 import _native, workloads
from forgetune_b200.autotuner import Autotuner, GpuCandidate
from forgetune_b200.frontend import export_to_ir
from forgetune_b200.graph_blob import serialize, tuning_of, with_tuning


def tiny_blob(max_batch=4096):
    ir = export_to_ir(workloads.tiny_mlp(), (torch.randn(2, 784),), True, max_batch)
    return serialize(ir, enable_fusion=True, bias_first_fused=True)


def test_candidate_space_contract():
    t = Autotuner()
    full = t.get_candidate_space()
    assert len(full) == 8 and full[0].candidate_id == "engine_default" and full[0].simplicity == 0
    assert [c.candidate_id for c in t.get_candidate_space(3)] == [c.candidate_id for c in full[:3]]
    assert all(not c.fuse_head for c in t.get_candidate_space(enable_fusion=False))
    assert all(c.fuse_head for c in t.get_candidate_space(force_fusion=True))
    assert any(not c.fuse_head for c in full)
    for bad in (0, 9, True, 2.0):
        with pytest.raises(ValueError):
            t.get_candidate_space(bad)
    with pytest.raises(ValueError):
        t.get_candidate_space(enable_fusion=False, force_fusion=True)
    assert [c.to_dict() for c in t.get_candidate_space()] == [c.to_dict() for c in full]  # deterministic


def test_selection_rules():
    t = Autotuner()
    cands = {c.candidate_id: c for c in t.get_candidate_space()}
    base = "engine_default"
    # under 5 %: the baseline stays
    assert t.select({base: 1.0, "tc_pair_k16": 0.96, "simt_ffma": 1.2}, cands, base)[0] == base
    # a clear winner
    assert t.select({base: 1.0, "tc_pair_k16": 0.5, "tc_sm_k16": 0.9}, cands, base)[0] == "tc_pair_k16"
    # two within 5 % of the fastest: the simpler one (tc_sm_k16, simplicity 1 < 2)
    assert t.select({base: 1.0, "tc_pair_k16": 0.50, "tc_sm_k16": 0.52}, cands, base)[0] == "tc_sm_k16"
    # outside the tie band the faster one wins even if less simple
    assert t.select({base: 1.0, "tc_pair_k16": 0.50, "tc_sm_k16": 0.60}, cands, base)[0] == "tc_pair_k16"


def test_batch_ranges_cover_and_merge():
    t = Autotuner()
    for batches, mx in (([1, 16, 256, 4096, 65536], 65536), ([7], 100), ([1, 2, 3], 3), ([16, 512], 4096)):
        r = t.buckets(batches, mx)
        assert r[0][0] == 1 and r[-1][1] == mx
        for (a0, a1), (b0, b1) in zip(r, r[1:]):
            assert b0 == a1 + 1 and a0 <= a1
        for b, (lo, hi) in zip(sorted(batches), r):
            assert lo <= b <= hi
    assert t.timing_batches(True, 65536, 1, 784, 10) == [1, 16, 256, 4096, 65536]
    assert t.timing_batches(False, 64, 64, 784 * 64, 640) == [64]
    with pytest.raises(ValueError):
        t.timing_batches(True, 100, 1, 784, 10, [200])
    # adjacent ranges with the same choice merge into one record per step
    cands = {c.candidate_id: c for c in t.get_candidate_space()}
    chosen = {(0, 0): "engine_default", (0, 1): "tc_pair_k16", (0, 2): "tc_pair_k16"}
    table = t._table([[0]], [(1, 4), (5, 64), (65, 1024)], chosen, cands, "engine_default")
    assert table == [[0, 5, 1024, 3, 0, 16, 0, 2, 1]]


def test_tuning_table_in_the_blob_and_its_validation():
    blob = tiny_blob()
    table = [[0, 1, 4096, 3, 256, 16, 1, 2, 1], [1, 17, 4096, 1, 0, 0, 0, 0, 1]]
    tuned = with_tuning(blob, table)
    assert tuning_of(tuned) == table and tuning_of(blob) == []
    assert with_tuning(tuned, []) == blob
    desc = _native.describe_blob(tuned)
    assert desc["steps"][0]["tuned"] == [[1, 4096, 3, 256, 16, 1, 2, 1]]
    assert desc["steps"][1]["head_step"] == 2 and desc["steps"][2]["head_of"] == 1
    bad = [[0, 5, 4, 3, 0, 0, 0, 0, 1],      # lo > hi
           [0, 1, 4, 7, 0, 0, 0, 0, 1],      # unknown family
           [0, 1, 4, 3, 96, 0, 0, 0, 1],     # tile width
           [0, 1, 4, 3, 64, 0, 0, 2, 1],     # SM-pair tiles of 64 columns
           [9, 1, 4, 3, 0, 0, 0, 0, 1]]      # no such step
    for rec in bad:
        with pytest.raises(Exception):
            _native.describe_blob(with_tuning(blob, [rec]))


def test_set_tuning_abi_validates_without_a_gpu():
    eng = _native.EngineModel(tiny_blob())
    eng.set_tuning([[0, 1, 100, 3, 0, 16, 0, 2, 1]])
    assert eng.describe()["steps"][0]["tuned"] == [[1, 100, 3, 0, 16, 0, 2, 1]]
    for rec in ([0, 1, 100, 3, 0, 16, 0, 2],):
        with pytest.raises(ValueError):
            eng.set_tuning([rec])
    with pytest.raises(Exception):
        eng.set_tuning([[5, 1, 100, 3, 0, 16, 0, 2, 1]])
    # a rejected table leaves the previous one in place
    assert eng.describe()["steps"][0]["tuned"] == [[1, 100, 3, 0, 16, 0, 2, 1]]
    eng.set_tuning([])
    assert all(s["tuned"] == [] for s in eng.describe()["steps"])
    L = _native.lib()
    assert L.ftb_model_set_tuning(None, None, 0) == -1
    assert L.ftb_model_set_tuning(eng.handle, None, 1) == -1
    assert L.ftb_model_set_tuning(eng.handle, ctypes.c_void_p(0), -1) == -6
    eng.close()


def test_candidate_records():
    c = GpuCandidate("x", 3, 128, 16, 1, 2, False, 2)
    assert c.record(4, 10, 20) == [4, 10, 20, 3, 128, 16, 1, 2, 0]
    with pytest.raises(ValueError):
        GpuCandidate("y", 9)
