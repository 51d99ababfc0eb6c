"""C-ABI behaviour on the GPU, mirroring the reference's acceptance suites
(tests/acceptance/test_v2_adversarial_boundary.py and
test_runtime_abi_robustness.py): batch boundaries, rejection, both entry
points, re-entrancy, multi-threading, zero steady-state allocation and
injected-allocation detection, all through the compiled model's C ABI."""

import concurrent.futures
import ctypes

import numpy as np
import pytest
import torch
import torch.nn as nn

from forgetune_b200 import InvalidShapeError, compile_model

pytestmark = pytest.mark.gpu


class LinearReLU(nn.Module):
    def __init__(self):
        super().__init__()
        self.fc = nn.Linear(8, 4)

    def forward(self, x):
        return torch.relu(self.fc(x))


@pytest.fixture(scope="module")
def dyn(tmp_path_factory):
    torch.manual_seed(42)
    m = LinearReLU().eval()
    cm = compile_model(m, (torch.randn(2, 8),), output_dir=str(tmp_path_factory.mktemp("dyn")), autotune=False,
                       dynamic_batch=True)
    yield cm, m
    cm.close()


@pytest.fixture(scope="module")
def static(tmp_path_factory):
    torch.manual_seed(42)
    m = LinearReLU().eval()
    cm = compile_model(m, (torch.randn(2, 8),), output_dir=str(tmp_path_factory.mktemp("st")), autotune=False,
                       dynamic_batch=False)
    yield cm, m
    cm.close()


def ref(m, x):
    with torch.no_grad():
        return m(torch.as_tensor(x)).numpy()


def test_boundary_batches(dyn, tmp_path):
    cm, m = dyn
    for b in [1, 2, 7, 16, 32, 64, 128]:
        x = torch.randn(b, 8)
        np.testing.assert_allclose(cm.run(x), ref(m, x), atol=1e-4, rtol=1e-4)
    cm300 = compile_model(m, (torch.randn(2, 8),), output_dir=str(tmp_path), autotune=False, dynamic_batch=True,
                          max_batch_size=300)
    for b in [1, 2, 150, 255, 256, 257, 300]:
        x = torch.randn(b, 8)
        np.testing.assert_allclose(cm300.run(x), ref(m, x), atol=1e-4, rtol=1e-4)
    with pytest.raises(InvalidShapeError):
        cm300.run(np.ones((301, 8), np.float32))
    cm300.close()


def test_dual_abi(dyn, static):
    for cm, _ in (dyn, static):
        rt = cm._runtime
        x = np.ones((2, 8), np.float32)
        y = np.zeros((2, 4), np.float32)
        xp = x.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
        yp = y.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
        assert rt.run_v1_fn(xp, 16, yp, 8) == 0
        assert rt.run_v2_fn(xp, 16, yp, 8, 2) == 0
        assert rt.run_v1_fn(None, 16, yp, 8) == -1
    assert dyn[0]._runtime.lib.forgetune_max_batch() == 128
    assert static[0]._runtime.lib.forgetune_max_batch() == 2


def test_numerical_stress(dyn):
    cm, m = dyn
    for x in (torch.zeros(5, 8), -100.0 * torch.ones(3, 8), 1e4 * torch.randn(9, 8)):
        np.testing.assert_allclose(cm.run(x), ref(m, x), atol=1e-4, rtol=1e-4)
    nan = torch.full((2, 8), float("nan"))
    assert np.isnan(cm.run(nan)).all()  # ReLU keeps NaN


def test_unaligned_input(dyn):
    cm, m = dyn
    buf = np.zeros(2 * 8 + 1, np.float32)
    x = buf[1:].reshape(2, 8)
    x[:] = 0.5
    assert x.ctypes.data % 16 != 0
    np.testing.assert_allclose(cm.run(x), ref(m, x.copy()), atol=1e-4, rtol=1e-4)


def test_alternating_batches(dyn):
    cm, m = dyn
    for b in [1, 64, 3, 128, 2, 16, 1, 32, 7, 64, 1]:
        x = torch.randn(b, 8)
        np.testing.assert_allclose(cm.run(x), ref(m, x), atol=1e-4, rtol=1e-4)


def test_same_thread_reentrancy(dyn):
    cm, m = dyn
    rt = cm._runtime
    x = np.ascontiguousarray(torch.randn(4, 8).numpy())
    y = np.zeros((4, 4), np.float32)
    for b in [1, 2, 7, 16]:
        xi = torch.randn(b, 8)
        np.testing.assert_allclose(cm.run(xi), ref(m, xi), atol=1e-4, rtol=1e-4)
    assert rt.run_v2_fn(x.ctypes.data, 32, y.ctypes.data, 16, 4) == 0
    np.testing.assert_allclose(y, ref(m, x), atol=1e-4, rtol=1e-4)


def test_concurrent_threads(dyn):
    cm, m = dyn

    def worker(tid):
        rng = np.random.default_rng(42 + tid)
        for _ in range(25):
            b = int(rng.choice([1, 2, 4, 7, 16, 32, 64]))
            x = rng.standard_normal((b, 8)).astype(np.float32)
            np.testing.assert_allclose(cm.run(x), ref(m, x), atol=1e-4, rtol=1e-4)
        return True

    with concurrent.futures.ThreadPoolExecutor(max_workers=8) as ex:
        assert all(f.result() for f in [ex.submit(worker, i) for i in range(8)])


def test_zero_allocation_steady_state(dyn):
    cm, m = dyn
    cm.run(torch.randn(1, 8))
    cm.reset_arena_alloc_count()
    assert cm.get_arena_alloc_count() == 0
    for b in [2, 7, 16, 32, 64, 128, 1, 16]:
        x = torch.randn(b, 8)
        np.testing.assert_allclose(cm.run(x), ref(m, x), atol=1e-4, rtol=1e-4)
    assert cm.get_arena_alloc_count() == 0
    assert cm.get_arena_payload_alloc_count() == 0
    assert cm.get_arena_block_insertion_count() == 0


def test_injected_allocation_detected_and_thread_isolation(dyn):
    cm, _ = dyn
    x1 = torch.randn(1, 8)
    cm.run(x1)
    cm.reset_arena_alloc_count()
    cm.run(x1)
    assert cm.get_arena_alloc_count() == 0
    cm.inject_test_arena_alloc()
    assert cm.get_arena_alloc_count() > 0
    assert cm.get_arena_payload_alloc_count() > 0
    cm.reset_arena_alloc_count()
    cm.run(x1)
    assert cm.get_arena_alloc_count() == 0

    def worker():
        cm.reset_arena_alloc_count()
        assert cm.get_arena_alloc_count() == 0
        cm.run(torch.randn(2, 8))
        allocs = cm.get_arena_alloc_count()
        cm.reset_arena_alloc_count()
        cm.run(torch.randn(4, 8))
        assert cm.get_arena_alloc_count() == 0
        return allocs

    with concurrent.futures.ThreadPoolExecutor(max_workers=1) as ex:
        assert ex.submit(worker).result() > 0
    assert cm.get_arena_alloc_count() == 0
    assert cm._runtime.get_process_arena_total_allocations() > 0


def test_benchmark_kernel_and_stress(dyn):
    cm, m = dyn
    us = cm.benchmark_kernel(iters=200, batch_size=64)
    assert 0 < us < 10000
    x = torch.randn(16, 8)
    want = ref(m, x)
    for _ in range(1000):
        got = cm.run(x)
    np.testing.assert_allclose(got, want, atol=1e-4, rtol=1e-4)


def test_close_and_reload(dyn, tmp_path):
    _, m = dyn
    cm = compile_model(m, (torch.randn(2, 8),), output_dir=str(tmp_path), autotune=False, dynamic_batch=True)
    x = torch.randn(3, 8)
    a = cm.run(x)
    cm._runtime.create()
    cm.close()
    with pytest.raises(Exception):
        cm.run(x)
    cm2 = compile_model(m, (torch.randn(2, 8),), output_dir=str(tmp_path), autotune=False, dynamic_batch=True)
    np.testing.assert_array_equal(cm2.run(x), a)
    cm2.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_in_process_sharding_over_devices(dyn, tmp_path):
    _, m = dyn
    cm = compile_model(m, (torch.randn(2, 8),), output_dir=str(tmp_path), autotune=False, dynamic_batch=True,
                       devices=[0, 1], max_batch_size=1000)
    x = torch.randn(999, 8)
    np.testing.assert_allclose(cm.run(x), ref(m, x), atol=1e-4, rtol=1e-4)
    cm.close()
