"""The CPU oracle is pinned to the reference runtime's own outputs.

golden.npz / golden.json hold outputs of the reference's generated runtime
(tests/golden/make_golden.py).  The oracle must reproduce them bit for bit for
both accumulation orders, and the seeded inputs must still hash to the values
recorded when the vectors were made.
"""
import hashlib
import json
import os

import numpy as np
import pytest
import torch

from forgetune_b200 import workloads
from oracle import oracle
from tests.golden.make_golden import make_input, sha, weights_sha

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
META = json.load(open(os.path.join(HERE, "golden.json")))
GOLD = np.load(os.path.join(HERE, "golden.npz"))
_MODELS = {}


def model(name):
    if name not in _MODELS:
        _MODELS[name] = workloads.WORKLOADS[name][0]()
    return _MODELS[name]


@pytest.mark.parametrize("name", sorted(META["weights_sha256"]))
def test_weights_match_golden(name):
    assert weights_sha(model(name)) == META["weights_sha256"][name]


CASES = [(c["key"], v) for c in META["cases"] for v in c["outputs"] if c["batch"] <= 4096]


@pytest.mark.parametrize("key,variant", CASES)
def test_oracle_bitwise_equals_reference(key, variant):
    case = next(c for c in META["cases"] if c["key"] == key)
    x = make_input(case["workload"], case["batch"], case["input"])
    assert sha(x) == case["input_sha256"], "seeded input drifted"
    y = oracle.run_model(model(case["workload"]), x, variant)
    assert sha(y) == case["outputs"][variant]["sha256"]
    np.testing.assert_array_equal(y.view(np.uint32), GOLD[key + "__" + variant].view(np.uint32))


def test_oracle_large_batch_sampled_rows():
    """B=65536 tiny-MLP sweep point: oracle on the sampled rows equals the stored rows."""
    case = next(c for c in META["cases"] if c["batch"] == 65536)
    rows = GOLD[case["key"] + "__rows"]
    x = make_input(case["workload"], case["batch"], case["input"])
    assert sha(x) == case["input_sha256"]
    for v in case["outputs"]:
        y = oracle.run_model(model(case["workload"]), x[rows], v)
        np.testing.assert_array_equal(y.view(np.uint32), GOLD[case["key"] + "__" + v].view(np.uint32))


def test_orders_differ_but_agree_within_tolerance():
    x = make_input("residual_mlp", 1024, "seeded")
    a = GOLD["residual_mlp_B1024_seeded__fused_ikj"]
    b = GOLD["residual_mlp_B1024_seeded__naive_ijk"]
    assert not np.array_equal(a, b)
    assert np.allclose(a, b, atol=1e-4, rtol=1e-4)
    del x


def test_philox_known_answer():
    """Philox4x32-10, counter 0 / key 0: the Random123 known-answer vector."""
    blk = oracle.philox_blocks(0, 0, 1)[0]
    assert [int(v) for v in blk] == [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]


def test_philox_normal_moments():
    z = oracle.philox_normal(1, 0, 1 << 18)
    assert abs(float(z.mean())) < 0.01
    assert abs(float(z.std()) - 1.0) < 0.01
    # counter-based: any window equals the same slice of a longer draw
    np.testing.assert_array_equal(oracle.philox_normal(1, 1000, 77), z[1000:1077])


def _float64_forward(m, x):
    h = x.astype(np.float64)
    for layer in m:
        if isinstance(layer, torch.nn.Linear):
            h = h @ layer.weight.detach().numpy().astype(np.float64).T + layer.bias.detach().numpy()
        else:
            h = np.maximum(h, 0.0)
    return h


def test_plain_tolerance_is_unattainable_at_wide_range():
    """At inputs x 1e3 the reference's fixed atol=1e-4 is below the rounding
    noise of fp32 arithmetic itself, so only the reference's own operation
    order can meet it: the reference's two variants (same k order, bias
    placed differently) fail allclose(1e-4, 1e-4) against each other on the
    residual MLP, and the exact float64 result fails it against the reference
    on the tiny MLP.  Both pass once atol is scaled with the input
    (atol = 1e-4 x 1e3), the criterion the GPU parity tests apply to the
    non-exact policies on these inputs."""
    a = GOLD["residual_mlp_B1024_wide_range__fused_ikj"]
    b = GOLD["residual_mlp_B1024_wide_range__naive_ijk"]
    assert not np.allclose(a, b, atol=1e-4, rtol=1e-4)
    assert np.allclose(a, b, atol=1e-4 * 1e3, rtol=1e-4)
    x = make_input("tiny_mlp", 4096, "wide_range")
    exact = _float64_forward(model("tiny_mlp"), x)
    ref = GOLD["tiny_mlp_B4096_wide_range__fused_ikj"]
    assert not np.allclose(exact, ref, atol=1e-4, rtol=1e-4)
    assert np.allclose(exact, ref, atol=1e-4 * 1e3, rtol=1e-4)
