#!/usr/bin/env python3
"""Throughput of the compiled forward pass: tiny MLP 784-256-128-10, global B=65536.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One process per GPU (torchrun for N > 1).  The global batch of 65536 rows is
split into contiguous row blocks, one per rank (strong scaling: 8192 rows per
GPU at N=8); each rank holds a weight replica and runs its block with no
collective on the data path.  Inputs are seeded N(0,1), generated on the
device by the counter-based Philox generator keyed by the global element
index, so a row's values do not depend on N.

value  device-resident samples/s over the global batch: K forward passes
       (one CUDA-graph replay each) on inputs already in HBM, each bracketed
       by CUDA events on the launching stream, with L2 flushed (a 256 MB write
       then read) before every step outside the events; the sum of the K
       intervals, max over ranks.
e2e    the same metric through the public host API (CompiledModel.run, the
       per-model library's forgetune_run_v2) on each rank's row block from
       pinned host memory, host<->device copies inside the timed region; wall
       clock around the synchronous calls, max over ranks.
extras (same JSON line) weak scaling (65536 rows per GPU) and the wide MLP
       (262144 rows split over the GPUs) at every N; at N=1 also the batch
       sweep B in {1, 8, 64, 128, 4096, 65536} (device time per forward and
       host-API p50), the residual MLP at B=1024 and the small CNN at B=256
       with their roofline fractions, and the CPU baseline.
--impl reference  the reference's own CPU runtime (the generated fused_ikj
       library built from the reference sources into oracle/_ref/) on every
       host core, one pinned thread per core: each step is one B=65536 pass
       split into contiguous row blocks.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import os
import queue
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

METRIC = "samples/sec (tiny MLP 784-256-128-10, global B=65536 split over the GPUs)"
UNIT = "samples/s"
BATCH = 65536
IN_F, OUT_F = 784, 10
REF_SO = os.path.join(HERE, "oracle", "_ref", "tiny_mlp_fused_ikj.so")
WORKLOAD = "tiny_mlp_784_256_128_10_dynamic_batch"
SWEEP = (1, 8, 64, 128, 4096, 65536)
WIDE_ROWS = 262144


def env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def host_cpus() -> list:
    try:
        return sorted(os.sched_getaffinity(0))
    except AttributeError:
        return list(range(os.cpu_count() or 1))


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


# ---------------------------------------------------------------------------
# reference CPU runtime (oracle/_ref): one pinned worker thread per host CPU
# ---------------------------------------------------------------------------
class RefRuntime:
    def __init__(self, path: str):
        self.lib = ctypes.CDLL(path)
        self.fn = self.lib.forgetune_run_v2
        self.fn.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int64]
        self.fn.restype = ctypes.c_int

    def run(self, x: np.ndarray, y: np.ndarray) -> None:
        rc = self.fn(x.ctypes.data, x.size, y.ctypes.data, y.size, x.shape[0])
        if rc != 0:
            raise RuntimeError("reference runtime returned %d" % rc)


class PinnedPool:
    """Worker threads, each pinned to one host CPU (sched_setaffinity on the
    thread itself).  The reference runtime is single-threaded per call and
    thread-safe (thread-local arenas), so N workers make N concurrent calls;
    ctypes releases the GIL around each."""

    def __init__(self, cpus):
        self.cpus = list(cpus)
        self.jobs = [queue.Queue() for _ in self.cpus]
        self.done = queue.Queue()
        self.threads = [threading.Thread(target=self._work, args=(i,), daemon=True) for i in range(len(self.cpus))]
        for t in self.threads:
            t.start()

    def _work(self, i):
        try:
            os.sched_setaffinity(0, {self.cpus[i]})
        except (AttributeError, OSError):
            pass
        while True:
            fn = self.jobs[i].get()
            if fn is None:
                return
            try:
                fn()
                self.done.put(None)
            except Exception as e:  # reported to the caller
                self.done.put(e)

    def run(self, fns) -> None:
        """fns[i] runs on worker i; returns when all have finished."""
        for i, fn in enumerate(fns):
            self.jobs[i].put(fn)
        errs = [self.done.get() for _ in fns]
        errs = [e for e in errs if e is not None]
        if errs:
            raise errs[0]

    def close(self):
        for q in self.jobs:
            q.put(None)


def split_pass(pool: PinnedPool, ref: RefRuntime, x: np.ndarray, y: np.ndarray) -> None:
    """One pass over x: contiguous row blocks, one call per worker."""
    n = len(pool.cpus)
    per = (x.shape[0] + n - 1) // n
    fns = []
    for r0 in range(0, x.shape[0], per):
        r1 = min(x.shape[0], r0 + per)
        fns.append(lambda a=r0, b=r1: ref.run(x[a:b], y[a:b]))
    pool.run(fns)


def one_core_rate(ref: RefRuntime, x: np.ndarray, seconds: float) -> float:
    """Samples/s of one pinned thread calling the reference on 2048-row blocks."""
    pool = PinnedPool(host_cpus()[:1])
    rows = 2048
    y = np.empty((rows, OUT_F), np.float32)
    xs = np.ascontiguousarray(x[:rows])
    pool.run([lambda: ref.run(xs, y)])  # warm-up: sizes the thread's arena
    done, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        pool.run([lambda: ref.run(xs, y)])
        done += rows
    rate = done / (time.perf_counter() - t0)
    pool.close()
    return rate


def cpu_baseline(passes: int = 4) -> dict:
    """Reference runtime on a bounded sample of the workload: `passes` full
    B=65536 passes on all host CPUs (one pinned thread each, contiguous row
    blocks: the procedure of --impl reference), and one pinned core on
    2048-row blocks for about 2 s."""
    if not os.path.isfile(REF_SO):
        return {"value": None, "unit": UNIT, "cores": 0, "kind": "reference",
                "sample": "unavailable: oracle/_ref not built"}
    from forgetune_b200 import workloads
    cpus = host_cpus()
    x = workloads.seeded_input((BATCH, IN_F)).numpy()
    y = np.empty((BATCH, OUT_F), np.float32)
    ref = RefRuntime(REF_SO)
    pool = PinnedPool(cpus)
    split_pass(pool, ref, x, y)  # warm-up: sizes every thread's arena
    t0 = time.perf_counter()
    for _ in range(passes):
        split_pass(pool, ref, x, y)
    dt = time.perf_counter() - t0
    pool.close()
    one = one_core_rate(ref, x, 2.0)
    return {"value": BATCH * passes / dt, "unit": UNIT, "cores": len(cpus), "kind": "reference",
            "cpu_model": cpu_model(), "one_core": {"value": one, "unit": UNIT, "cores": 1},
            "sample": "%d full B=65536 passes on %d pinned threads (contiguous row blocks, one ctypes call per "
                      "thread) in %.2f s; one core: one pinned thread on 2048-row blocks for 2 s; reference "
                      "fused_ikj runtime built from the reference sources" % (passes, len(cpus), dt)}


def run_reference(args) -> int:
    rank = env_int("RANK", 0)
    if rank != 0:
        return 0
    if not os.path.isfile(REF_SO):
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/tiny_mlp_fused_ikj.so not built "
                                                                "(python oracle/build_ref.py)"}))
        return 0
    from forgetune_b200 import workloads
    cpus = host_cpus()
    x = workloads.seeded_input((BATCH, IN_F)).numpy()
    y = np.empty((BATCH, OUT_F), np.float32)
    ref = RefRuntime(REF_SO)
    pool = PinnedPool(cpus)
    for _ in range(args.warmup):
        split_pass(pool, ref, x, y)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        split_pass(pool, ref, x, y)
        times.append(time.perf_counter() - t0)
    pool.close()
    total = sum(times)
    value = BATCH * args.steps / total
    one = one_core_rate(ref, x, 2.0)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * total / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "global_batch": BATCH, "threads": len(cpus)},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": len(cpus), "kind": "reference",
                         "cpu_model": cpu_model(), "one_core": {"value": one, "unit": UNIT, "cores": 1},
                         "sample": "full B=65536 pass per step on %d pinned threads (contiguous row blocks); "
                                   "one core: one pinned thread on 2048-row blocks for 2 s" % len(cpus)},
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


def model_flops(model, sample_shape) -> float:
    """FLOPs of one sample's forward pass: 2 per multiply-add of every Linear
    and Conv2d (shapes from a CPU forward with hooks)."""
    import torch
    total = [0.0]

    def hook(mod, inp, out):
        if isinstance(mod, torch.nn.Linear):
            total[0] += 2.0 * mod.in_features * mod.out_features
        elif isinstance(mod, torch.nn.Conv2d):
            kh, kw = mod.kernel_size
            total[0] += 2.0 * out[0].numel() * (mod.in_channels // mod.groups) * kh * kw

    hs = [m.register_forward_hook(hook) for m in model.modules() if isinstance(m, (torch.nn.Linear, torch.nn.Conv2d))]
    with torch.no_grad():
        model(torch.zeros((1,) + tuple(sample_shape)))
    for h in hs:
        h.remove()
    return total[0]


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
class Timer:
    """Per-step CUDA events on the launching stream with an L2 flush (256 MB
    written, then read) before each step, outside the events."""

    def __init__(self, dev, stream):
        import torch
        self.torch = torch
        self.stream = stream
        self.buf = torch.empty(64 << 20, dtype=torch.float32, device=dev)
        self.sink = torch.empty((), dtype=torch.float32, device=dev)

    def flush(self):
        self.buf.zero_()
        self.torch.sum(self.buf, dim=0, out=self.sink)

    def run(self, step, iters):
        """Durations (ms) of `iters` calls of step(i), each after a flush."""
        torch = self.torch
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters)]
        for i in range(iters):
            self.flush()
            ev[i][0].record(self.stream)
            step(i)
            ev[i][1].record(self.stream)
        torch.cuda.synchronize()
        return [a.elapsed_time(b) for a, b in ev]


def build_engine(model, sample_shape, max_batch, dev_index, policy="auto"):
    """The compiled graph (the blob compile_model embeds) as an engine handle."""
    import torch
    from forgetune_b200 import _native
    from forgetune_b200.frontend import export_to_ir
    from forgetune_b200.graph_blob import serialize
    x = torch.zeros((2,) + tuple(sample_shape))
    ir = export_to_ir(model, (x,), dynamic_batch=True, max_batch_size=max_batch)
    eng = _native.EngineModel(serialize(ir, enable_fusion=True, bias_first_fused=True, kernel_policy=policy))
    eng.set_devices([dev_index])
    eng.prepare()
    return eng


def forward_profile(eng, step_fn, timer, iters):
    """Per-launch-list-step device ms averaged over `iters` profiled runs."""
    for i in range(2):
        step_fn(i)
    import torch
    torch.cuda.synchronize()
    for i in range(iters):
        timer.flush()
        step_fn(i)
    torch.cuda.synchronize()
    return np.array([eng.profile_read(i) for i in range(iters)]).mean(axis=0)


def config_extra(name, builder, sample_shape, B, dev, stream, timer, peak_tflops, iters=20):
    """Device time per forward of a workload at batch B (graph replays, L2
    flushed before each), FLOPs and the roofline fraction of the forward and
    of its dominant launch."""
    import torch
    from forgetune_b200 import _native
    model = builder()
    eng = build_engine(model, sample_shape, B, dev.index)
    n_in = B * int(np.prod(sample_shape))
    out_f = int(model(torch.zeros((1,) + tuple(sample_shape))).shape[1])
    x = torch.empty(n_in, dtype=torch.float32, device=dev)
    y = torch.empty(B * out_f, dtype=torch.float32, device=dev)
    _native.philox_normal(x.data_ptr(), 1, 0, n_in, stream.cuda_stream)

    def step(i):
        eng.run_device(x.data_ptr(), n_in, y.data_ptr(), B * out_f, B, stream.cuda_stream)

    for i in range(3):
        step(i)
    ms = timer.run(step, iters)
    prof = forward_profile(eng, lambda i: eng.run_device_profiled(x.data_ptr(), n_in, y.data_ptr(), B * out_f, B,
                                                                  stream.cuda_stream, i), timer, iters)
    flops = model_flops(model, sample_shape) * B
    med = statistics.median(ms)
    dom = int(np.argmax(prof))
    st = eng.desc["steps"][dom]
    res = {"workload": name, "batch": B, "device_ms_median": med, "samples_per_s": B / (med / 1000.0),
           "flops_per_forward": flops, "tflops": flops / (med / 1000.0) / 1e12,
           "roofline_frac_forward": flops / (med / 1000.0) / 1e12 / peak_tflops,
           "kernels_per_forward": eng.graph_kernels(),
           "dominant_step": {"index": dom, "kind": st.get("kind"), "K": st.get("K"), "N": st.get("N"),
                             "avg_ms": float(prof[dom]), "share_of_forward": float(prof[dom] / prof.sum())},
           "per_step_ms": [round(float(v), 5) for v in prof],
           "l2": "flushed before each forward"}
    eng.close()
    return res


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

    G = args.batch  # global batch
    r0, r1 = sharding.shard_rows(G, world, rank)
    B = r1 - r0  # this rank's rows
    model = workloads.tiny_mlp()
    out_dir = tempfile.mkdtemp(prefix="ftb_bench_r%d_" % rank)
    cm = compile_model(model, (workloads.seeded_input((64, IN_F)),), output_dir=out_dir, autotune=False,
                       kernel_variant="fused_ikj", enable_fusion=True, dynamic_batch=True,
                       max_batch_size=max(B, BATCH),
                       max_workspace_bytes=8 << 30, gpu_kernel=args.policy)
    with open(cm.manifest()["artifacts"]["graph_blob"], "rb") as f:
        eng = _native.EngineModel(f.read())
    eng.set_devices([local])
    eng.prepare()
    steps_desc = eng.desc["steps"]

    stream = torch.cuda.current_stream(dev)
    timer = Timer(dev, stream)
    x = torch.empty(B * IN_F, dtype=torch.float32, device=dev)
    y = torch.empty(B * OUT_F, dtype=torch.float32, device=dev)
    _native.philox_normal(x.data_ptr(), 1, r0 * IN_F, B * IN_F, stream.cuda_stream)
    torch.cuda.synchronize()

    def step(i):
        # one replay of the forward's CUDA graph (the path the public API runs)
        eng.run_device(x.data_ptr(), B * IN_F, y.data_ptr(), B * OUT_F, B, stream.cuda_stream)

    def step_prof(i):
        # the same kernels launched with an event before every launch-list
        # step (about 3.5 us per event): each kernel's device time
        eng.run_device_profiled(x.data_ptr(), B * IN_F, y.data_ptr(), B * OUT_F, B, stream.cuda_stream, i % 1024)

    for i in range(args.warmup):
        timer.flush()
        step(i)
        step_prof(i)
    torch.cuda.synchronize()
    launches_per_step = eng.graph_kernels()
    barrier()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    torch.cuda.synchronize()
    barrier()
    # timed region 1 (the headline): K graph replays
    ms_steps = timer.run(step, args.steps)
    barrier()
    # timed region 2 (the roofline): the same K steps with per-kernel events
    prof_steps = timer.run(step_prof, args.steps)
    barrier()
    clk = clocks.stop()
    ms = max_over_ranks(sum(ms_steps))
    ms_prof = max_over_ranks(sum(prof_steps))
    value = G * args.steps / (ms / 1000.0)

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
    tc_peak = peaks["bf16_tflops"] / 6.0  # 3xTF32: three tf32 MMAs at half the bf16 rate
    flops = sum(2.0 * B * steps_desc[i]["K"] * steps_desc[i]["N"] for i in fused_steps)
    dom_ms = max_over_ranks(float(avg[dom]))
    achieved_tflops = flops / (dom_ms / 1000.0) / 1e12
    traffic, kname = None, ds.get("kernel", "")
    tpath = os.path.join(HERE, "profiles", "traffic.json")
    if os.path.isfile(tpath):
        with open(tpath) as f:
            rec = json.load(f).get(WORKLOAD, {}).get("rows_%d" % B, {})
        traffic = rec.get("dominant_kernel_bytes_per_launch")
        kname = kname or rec.get("dominant_kernel", "")
    roofline = {
        "bound": "tensor", "achieved": achieved_tflops, "peak": tc_peak, "unit": "TFLOP/s",
        "frac": achieved_tflops / tc_peak, "traffic": traffic,
        "kernel": "steps %s: GEMMs %s, M=%d (%s)" % (
            fused_steps, " + ".join("K=%d N=%d" % (steps_desc[i]["K"], steps_desc[i]["N"]) for i in fused_steps),
            B, kname),
        "algorithmic_flops_per_launch": flops, "avg_launch_ms": dom_ms,
        "timed_over": "a second timed region of the same %d steps with CUDA events between launch-list steps "
                      "(%.4f ms per step there, against %.4f ms per step without the events); max over ranks"
                      % (args.steps, ms_prof / args.steps, ms / args.steps),
        "share_of_forward": float(avg[dom] / avg.sum()),
        "peak_basis": "fp32-accurate contraction on tensor cores = 3xTF32 = %s bf16 dense / 6 (%.1f / 6)"
                      % (peaks["_source"], peaks["bf16_tflops"]),
        "forward_frac": (B * 469504.0 / (ms / args.steps / 1000.0) / 1e12) / tc_peak,
    }

    extras = {}
    # weak scaling: 65536 rows on every GPU (a larger global batch as N grows)
    if world > 1:
        xw = torch.empty(BATCH * IN_F, dtype=torch.float32, device=dev)
        yw = torch.empty(BATCH * OUT_F, dtype=torch.float32, device=dev)
        _native.philox_normal(xw.data_ptr(), 1, rank * BATCH * IN_F, BATCH * IN_F, stream.cuda_stream)

        def step_w(i):
            eng.run_device(xw.data_ptr(), BATCH * IN_F, yw.data_ptr(), BATCH * OUT_F, BATCH, stream.cuda_stream)

        for i in range(3):
            step_w(i)
        barrier()
        wms = max_over_ranks(sum(timer.run(step_w, args.steps)))
        extras["weak_scaling"] = {"rows_per_gpu": BATCH, "global_batch": BATCH * world,
                                  "value": BATCH * world * args.steps / (wms / 1000.0), "unit": UNIT,
                                  "ms_per_step": wms / args.steps}
        del xw, yw
    else:
        extras["weak_scaling"] = {"rows_per_gpu": BATCH, "global_batch": BATCH, "value": value, "unit": UNIT,
                                  "ms_per_step": ms / args.steps}

    e2e, base = None, None
    if not args.quick:
        # end to end through the public host API, pinned host buffers, this rank's row block
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
        e2e = {"value": G * args.steps / e2e_s, "unit": UNIT,
               "h2d_bytes_per_step": G * IN_F * 4, "d2h_bytes_per_step": G * OUT_F * 4,
               "h2d_bytes_per_step_per_gpu": B * IN_F * 4, "d2h_bytes_per_step_per_gpu": int(out_host.nbytes),
               "ms_per_step": 1000.0 * e2e_s / args.steps}
        e2e.update(host_link(xh, dev, stream, max_over_ranks, e2e["ms_per_step"]))
        del xh

        # wide MLP at box scale: 262144 rows split over the GPUs, generated per shard on the device
        extras["wide_mlp"] = wide_mlp_extra(world, rank, dev, stream, timer, tc_peak, max_over_ranks, barrier)

        if world == 1:
            extras["sweep"] = sweep_extra(cm, eng, dev, stream, timer, tc_peak)
            extras["residual_mlp"] = config_extra("residual_mlp_512x10_blocks", workloads.residual_mlp, (512,), 1024,
                                                  dev, stream, timer, tc_peak)
            extras["small_cnn"] = config_extra("small_cnn_3x32x32", workloads.small_cnn, (3, 32, 32), 256, dev,
                                               stream, timer, tc_peak)
            base = cpu_baseline() if rank == 0 else None
    if rank == 0:
        b1 = extras.get("sweep", {}).get("1", {})
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "global_batch": G, "rows_per_gpu": B,
                       "kernel_policy": args.policy, "parallelism": "contiguous row blocks, weight replica per GPU",
                       "l2": "flushed before every timed step (256 MB written, then read), outside the events"},
            "e2e": e2e,
            "gpu_launches": args.steps * launches_per_step,
            "roofline": roofline,
            "clocks": clk,
            "latency_b1": {"p50_host_api_us": b1.get("host_api_p50_us"), "device_us": b1.get("device_us_median")},
            "per_step_ms": [float(v) for v in avg],
            "extras": extras,
        }
        if base is not None:
            line["cpu_baseline"] = base
        print(json.dumps(line))
    eng.close()
    cm.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


def host_link(xh, dev, stream, max_over_ranks, e2e_ms: float) -> dict:
    """The host link's own speed for this step's input: one pinned-host ->
    device copy of the same bytes (cudaMemcpyAsync), timed with CUDA events
    over five copies after one warm-up, slowest rank.  The e2e step cannot
    beat it (the run path overlaps the output's copy and the compute with
    it), so link_bound_ms / e2e ms_per_step is e2e's fraction of the link."""
    import torch
    d = torch.empty(xh.shape, dtype=xh.dtype, device=dev)
    reps = 5
    with torch.cuda.stream(stream):
        d.copy_(xh, non_blocking=True)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(reps):
            d.copy_(xh, non_blocking=True)
        t1.record(stream)
    t1.synchronize()
    ms = max_over_ranks(t0.elapsed_time(t1) / reps)
    del d
    nbytes = xh.numel() * xh.element_size()
    return {"link_h2d_gbs": nbytes / (ms / 1000.0) / 1e9, "link_bound_ms": ms, "frac_of_link": ms / e2e_ms,
            "link_basis": "pinned host -> device copy of this step's input bytes, CUDA events, slowest rank"}


def sweep_extra(cm, eng, dev, stream, timer, tc_peak) -> dict:
    """Config-2 batch sweep: device time per forward (graph replay, L2 flushed
    before each, median of 30) and the public host API's p50 (pinned input)."""
    import torch
    from forgetune_b200 import _native
    out = {}
    xmax = torch.empty(max(SWEEP) * IN_F, dtype=torch.float32, device=dev)
    ymax = torch.empty(max(SWEEP) * OUT_F, dtype=torch.float32, device=dev)
    _native.philox_normal(xmax.data_ptr(), 1, 0, max(SWEEP) * IN_F, stream.cuda_stream)
    xh_all = torch.empty((max(SWEEP), IN_F), dtype=torch.float32, pin_memory=True)
    xh_all.copy_(xmax.view(-1, IN_F))
    rt = cm._runtime
    for b in SWEEP:
        def step(i, b=b):
            eng.run_device(xmax.data_ptr(), b * IN_F, ymax.data_ptr(), b * OUT_F, b, stream.cuda_stream)
        for i in range(3):
            step(i)
        ms = timer.run(step, 30)
        med = statistics.median(ms)
        xb = xh_all[:b].numpy()
        calls = 200 if b <= 4096 else 20
        for _ in range(10):
            rt.run(xb)
        lat = []
        for _ in range(calls):
            t0 = time.perf_counter_ns()
            rt.run(xb)
            lat.append((time.perf_counter_ns() - t0) / 1000.0)
        p50 = statistics.median(lat)
        flops = 2.0 * b * (784 * 256 + 256 * 128 + 128 * 10)
        out[str(b)] = {"device_us_median": med * 1000.0, "samples_per_s_device": b / (med / 1000.0),
                       "host_api_p50_us": p50, "samples_per_s_host_api": b / (p50 / 1e6),
                       "roofline_frac": flops / (med / 1000.0) / 1e12 / tc_peak,
                       "kernels_per_forward": eng.graph_kernels()}
    return out


def wide_mlp_extra(world, rank, dev, stream, timer, tc_peak, max_over_ranks, barrier) -> dict:
    """Config 5: 262144 rows split over the ranks, each shard generated on the
    device from the global element index; 1 warm-up + 3 timed forwards."""
    import torch
    from forgetune_b200 import _native, sharding, workloads
    r0, r1 = sharding.shard_rows(WIDE_ROWS, world, rank)
    B = r1 - r0
    model = workloads.wide_mlp()
    eng = build_engine(model, (4096,), B, dev.index)
    x = torch.empty(B * 4096, dtype=torch.float32, device=dev)
    y = torch.empty(B * 4096, dtype=torch.float32, device=dev)
    _native.philox_normal(x.data_ptr(), 1, r0 * 4096, B * 4096, stream.cuda_stream)

    def step(i):
        eng.run_device(x.data_ptr(), B * 4096, y.data_ptr(), B * 4096, B, stream.cuda_stream)

    step(0)
    torch.cuda.synchronize()
    barrier()
    ms = max_over_ranks(sum(timer.run(step, 3)))
    flops = 2.0 * WIDE_ROWS * (4096 * 8192 + 8192 * 8192 + 8192 * 4096)
    tflops = flops * 3 / (ms / 1000.0) / 1e12
    res = {"workload": "wide_mlp_4096_8192_8192_4096", "global_batch": WIDE_ROWS, "rows_per_gpu": B,
           "n_gpus": world, "steps": 3, "ms_per_step": ms / 3, "samples_per_s": WIDE_ROWS * 3 / (ms / 1000.0),
           "tflops_all_gpus": tflops, "roofline_frac_per_gpu": tflops / world / tc_peak,
           "kernels_per_forward": eng.graph_kernels(), "scaling": "strong"}
    eng.close()
    del x, y
    torch.cuda.empty_cache()
    return res


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=BATCH, help="global batch split over the ranks")
    ap.add_argument("--policy", default="auto", choices=["auto", "simt", "simt_exact", "tcgen05"])
    ap.add_argument("--quick", action="store_true",
                    help="device-resident timing only (no e2e, extras or CPU baseline), for profiler captures")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
