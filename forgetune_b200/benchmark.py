"""Host-side latency statistics (the reference's benchmark_function,
python/forgetune/benchmark.py:12-58: perf_counter_ns, median / IQR / p90 / p99)."""

from __future__ import annotations

import os
import platform
import time
from typing import Any, Callable, Dict

import numpy as np


def benchmark_function(fn: Callable[[], Any], warmup_iters: int = 10, measure_iters: int = 50) -> Dict[str, Any]:
    for _ in range(warmup_iters):
        fn()
    samples = np.empty(measure_iters, dtype=np.float64)
    for i in range(measure_iters):
        t0 = time.perf_counter_ns()
        fn()
        samples[i] = (time.perf_counter_ns() - t0) / 1000.0
    q = np.percentile(samples, [25, 50, 75, 90, 99])
    return {
        "median_us": float(q[1]),
        "mean_us": float(samples.mean()),
        "min_us": float(samples.min()),
        "max_us": float(samples.max()),
        "iqr_us": float(q[2] - q[0]),
        "p90_us": float(q[3]),
        "p99_us": float(q[4]),
        "samples": int(measure_iters),
    }


def get_machine_metadata() -> Dict[str, Any]:
    cpu = platform.processor() or ""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    cpu = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return {"cpu": cpu, "cores": os.cpu_count(), "platform": platform.platform()}
