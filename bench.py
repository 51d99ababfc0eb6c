#!/usr/bin/env python3
"""Throughput of the compiled forward pass: tiny MLP 784-256-128-10 at B=65536 per GPU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One process per GPU (torchrun for N > 1).  Each rank holds a weight replica
and processes its own 65536-row shard of a global batch (weak scaling: the
batch dimension shards with no collective).  Inputs are seeded N(0,1),
generated on the device by the counter-based Philox generator keyed by the
global element index, so a rank's shard does not depend on N.

value  device-resident samples/s: K forward passes on inputs already in HBM
       (205 MB input per pass, larger than the 126 MB L2, so no flush is
       needed), CUDA events on the launching stream, max over ranks.
e2e    the same metric through the public host API (CompiledModel.run, the
       per-model library's forgetune_run_v2) from pinned host memory, the
       host<->device copies inside the timed region; wall clock around
       synchronous calls, max over ranks.
--impl reference  the reference's own CPU runtime (the generated fused_ikj
       library built from the reference sources into oracle/_ref/) on all
       host cores: each step is one B=65536 pass split across threads.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

METRIC = "samples/sec (tiny MLP 784-256-128-10, B=65536 per GPU)"
UNIT = "samples/s"
BATCH = 65536
IN_F, OUT_F = 784, 10
REF_SO = os.path.join(HERE, "oracle", "_ref", "tiny_mlp_fused_ikj.so")
WORKLOAD = "tiny_mlp_784_256_128_10_dynamic_batch"


def env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# ---------------------------------------------------------------------------
# reference CPU runtime (oracle/_ref): all host threads, contiguous row slices
# ---------------------------------------------------------------------------
class RefRuntime:
    def __init__(self, path: str):
        self.lib = ctypes.CDLL(path)
        self.fn = self.lib.forgetune_run_v2
        self.fn.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int64]
        self.fn.restype = ctypes.c_int

    def run_split(self, x: np.ndarray, y: np.ndarray, threads: int) -> None:
        B = x.shape[0]
        per = (B + threads - 1) // threads
        errs = []

        def work(r0, r1):
            rc = self.fn(x[r0:r1].ctypes.data, (r1 - r0) * IN_F, y[r0:r1].ctypes.data, (r1 - r0) * OUT_F, r1 - r0)
            if rc != 0:
                errs.append(rc)

        ts = [threading.Thread(target=work, args=(r0, min(B, r0 + per))) for r0 in range(0, B, per)]
        for t in ts:
            t.start()
        for t in ts:
            t.join()
        if errs:
            raise RuntimeError("reference runtime returned %s" % errs)


def cpu_baseline(seconds: float = 1.5) -> dict:
    """Reference runtime on every host thread over a bounded sample of the workload."""
    if not os.path.isfile(REF_SO):
        return {"value": None, "unit": UNIT, "cores": 0, "kind": "reference",
                "sample": "unavailable: oracle/_ref not built"}
    from forgetune_b200 import workloads
    threads = cpu_threads()
    rows = min(BATCH, max(threads * 256, 4096))
    x = workloads.seeded_input((rows, IN_F)).numpy()
    y = np.empty((rows, OUT_F), np.float32)
    ref = RefRuntime(REF_SO)
    ref.run_split(x, y, threads)  # warm-up: sizes every thread's arena
    done, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        ref.run_split(x, y, threads)
        done += rows
    dt = time.perf_counter() - t0
    return {"value": done / dt, "unit": UNIT, "cores": threads, "kind": "reference",
            "sample": "%d-row slices of the seeded B=65536 input, %d passes over %.1f s wall "
                      "(%.0f CPU-seconds), reference fused_ikj runtime, one ctypes call per thread"
                      % (rows, done // rows, dt, dt * threads)}


def run_reference(args) -> int:
    rank = env_int("RANK", 0)
    if rank != 0:
        return 0
    if not os.path.isfile(REF_SO):
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/tiny_mlp_fused_ikj.so not built "
                                                                "(python oracle/build_ref.py)"}))
        return 0
    from forgetune_b200 import workloads
    threads = cpu_threads()
    x = workloads.seeded_input((BATCH, IN_F)).numpy()
    y = np.empty((BATCH, OUT_F), np.float32)
    ref = RefRuntime(REF_SO)
    for _ in range(args.warmup):
        ref.run_split(x, y, threads)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        ref.run_split(x, y, threads)
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = BATCH * args.steps / total
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * total / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "batch_per_step": BATCH, "threads": threads},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "reference",
                         "sample": "full B=65536 pass per step split over %d threads" % threads},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    return 0


# ---------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device), "--query-gpu=" + self.FIELDS,
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons, power = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [v.strip() for v in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
                power.append(float(f[3]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm), "power_w_max": max(power) if power else None}


def load_peaks() -> dict:
    p = os.path.join(HERE, "MEASURED_PEAKS.json")
    if os.path.isfile(p):
        with open(p) as f:
            d = json.load(f)
        d["_source"] = "measured"
        return d
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "_source": "fallback"}


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def run_ours(args) -> int:
    import torch
    import torch.distributed as dist

    from forgetune_b200 import _native, compile_model, sharding, workloads

    rank, world, local = sharding.rank_info()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        sharding.init("nccl", dev)
    barrier = sharding.barrier

    def max_over_ranks(v: float) -> float:
        return sharding.max_over_ranks(v, dev)

    B = args.batch
    model = workloads.tiny_mlp()
    out_dir = tempfile.mkdtemp(prefix="ftb_bench_r%d_" % rank)
    cm = compile_model(model, (workloads.seeded_input((64, IN_F)),), output_dir=out_dir, autotune=False,
                       kernel_variant="fused_ikj", enable_fusion=True, dynamic_batch=True, max_batch_size=B,
                       max_workspace_bytes=8 << 30, gpu_kernel=args.policy)
    with open(cm.manifest()["artifacts"]["graph_blob"], "rb") as f:
        eng = _native.EngineModel(f.read())
    eng.set_devices([local])
    eng.prepare()
    steps_desc = eng.desc["steps"]

    stream = torch.cuda.current_stream(dev)
    x = torch.empty(B * IN_F, dtype=torch.float32, device=dev)
    y = torch.empty(B * OUT_F, dtype=torch.float32, device=dev)
    _native.philox_normal(x.data_ptr(), 1, sharding.shard_element_offset(rank, B, IN_F), B * IN_F,
                          stream.cuda_stream)
    torch.cuda.synchronize()

    def step(slot=None):
        # a step is one replay of the forward's CUDA graph (the path the public
        # API runs); profiled steps launch the same kernels with an event
        # before every launch-list step, which costs about 3.5 us per event
        if slot is None:
            eng.run_device(x.data_ptr(), B * IN_F, y.data_ptr(), B * OUT_F, B, stream.cuda_stream)
        else:
            eng.run_device_profiled(x.data_ptr(), B * IN_F, y.data_ptr(), B * OUT_F, B, stream.cuda_stream, slot)

    for i in range(args.warmup):
        step()
        step(i % 1024)
    torch.cuda.synchronize()
    launches_per_step = eng.graph_kernels()
    barrier()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    torch.cuda.synchronize()
    barrier()

    def timed(profiled):
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        for i in range(args.steps):
            step(i % 1024 if profiled else None)
        ev1.record(stream)
        torch.cuda.synchronize()
        return ev0.elapsed_time(ev1)

    # timed region 1 (the headline): K graph replays, nothing else on the stream
    ms_local = timed(False)
    barrier()
    # timed region 2 (the roofline): the same K steps with per-step events,
    # giving each kernel's device time
    ms_prof_local = timed(True)
    barrier()
    clk = clocks.stop()
    ms = max_over_ranks(ms_local)
    ms_prof = max_over_ranks(ms_prof_local)
    value = world * B * args.steps / (ms / 1000.0)

    # per-step device times from the events recorded inside timed region 2
    nprof = min(args.steps, 1024)
    per_step = np.array([eng.profile_read(i) for i in range(nprof)])
    avg = per_step.mean(axis=0)
    dom = int(np.argmax(avg))
    ds = steps_desc[dom]
    # the steps the dominant launch computes: with one launch per forward the
    # two-layer kernel also ran the second layer and its head
    fused_steps = [dom]
    if ds.get("mlp_step", -1) >= 0 and launches_per_step == 1:
        fused_steps.append(ds["mlp_step"])
        if steps_desc[ds["mlp_step"]].get("head_step", -1) >= 0:
            fused_steps.append(steps_desc[ds["mlp_step"]]["head_step"])
    peaks = load_peaks()
    flops = sum(2.0 * B * steps_desc[i]["K"] * steps_desc[i]["N"] for i in fused_steps)
    achieved_tflops = flops / (avg[dom] / 1000.0) / 1e12
    tc_peak = peaks["bf16_tflops"] / 6.0  # 3xTF32: three tf32 MMAs at half the bf16 rate
    traffic, kname = None, ds.get("kernel", "")
    tpath = os.path.join(HERE, "profiles", "traffic.json")
    if os.path.isfile(tpath):
        with open(tpath) as f:
            rec = json.load(f).get(WORKLOAD, {})
        traffic = rec.get("dominant_kernel_bytes_per_launch")
        kname = kname or rec.get("dominant_kernel", "")
    roofline = {
        "bound": "tensor", "achieved": achieved_tflops, "peak": tc_peak, "unit": "TFLOP/s",
        "frac": achieved_tflops / tc_peak, "traffic": traffic,
        "kernel": "steps %s: GEMMs %s, M=%d (%s)" % (
            fused_steps, " + ".join("K=%d N=%d" % (steps_desc[i]["K"], steps_desc[i]["N"]) for i in fused_steps),
            B, kname),
        "algorithmic_flops_per_launch": flops, "avg_launch_ms": float(avg[dom]),
        "timed_over": "a second timed region of the same %d steps with CUDA events between launch-list steps "
                      "(%.4f ms per step there, against %.4f ms per step without the events)"
                      % (args.steps, ms_prof / args.steps, ms / args.steps),
        "share_of_forward": float(avg[dom] / avg.sum()),
        "peak_basis": "fp32-accurate contraction on tensor cores = 3xTF32 = %s bf16 dense / 6 (%.0f / 6)"
                      % (peaks["_source"], peaks["bf16_tflops"]),
        "fp32_ffma_nominal_tflops": 148 * 128 * 2 * 1.965e9 / 1e12,
    }

    e2e, p50_b1, dev_b1, base = None, None, None, None
    if not args.quick:
        # end to end through the public host API, pinned host buffers
        xh = torch.empty((B, IN_F), dtype=torch.float32, pin_memory=True)
        xh.copy_(x.view(B, IN_F))
        xh_np = xh.numpy()
        rt = cm._runtime
        for _ in range(max(1, args.warmup)):
            rt.run(xh_np)
        barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            out_host = rt.run(xh_np)
        e2e_s = max_over_ranks(time.perf_counter() - t0)
        e2e = {"value": world * B * args.steps / e2e_s, "unit": UNIT,
               "h2d_bytes_per_step": B * IN_F * 4, "d2h_bytes_per_step": int(out_host.nbytes),
               "ms_per_step": 1000.0 * e2e_s / args.steps}

        # p50 latency at B=1 through the host API (graph replay)
        x1 = np.ascontiguousarray(xh_np[:1])
        for _ in range(20):
            rt.run(x1)
        lat = []
        for _ in range(200):
            t0 = time.perf_counter_ns()
            rt.run(x1)
            lat.append((time.perf_counter_ns() - t0) / 1000.0)
        p50_b1 = statistics.median(lat)
        dev_b1 = cm.benchmark_kernel(iters=1000, batch_size=1)
        base = cpu_baseline() if (rank == 0 and world == 1) else None
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "batch_per_gpu": B, "global_batch": B * world,
                       "kernel_policy": args.policy, "parallelism": "batch shards, weight replica per GPU",
                       "l2": "input 205 MB per pass > 126 MB L2; no flush"},
            "e2e": e2e,
            "gpu_launches": args.steps * launches_per_step,
            "roofline": roofline,
            "clocks": clk,
            "latency_b1": {"p50_host_api_us": p50_b1, "device_us": dev_b1},
            "per_step_ms": [float(v) for v in avg],
        }
        if base is not None:
            line["cpu_baseline"] = base
        print(json.dumps(line))
    eng.close()
    cm.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=BATCH)
    ap.add_argument("--policy", default="auto", choices=["auto", "simt", "simt_exact", "tcgen05"])
    ap.add_argument("--quick", action="store_true",
                    help="device-resident timing only (no e2e, latency or CPU baseline), for profiler captures")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
