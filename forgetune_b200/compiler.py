"""Public API: ``compile_model`` and ``CompiledModel``.

Same entry point, keyword arguments, validation and return type as the
reference (python/forgetune/compiler.py:381-794).  The pipeline is

  1. torch.export -> reference IR (frontend.py)
  2. graph blob with the weights (graph_blob.py)
  3. fusion + arena plan by the native engine; workspace budget check
     (the reference's MemoryPlanner check, compiler.py:647-658)
  4. per-model shim emitted and built with the host compiler (emit.py)
  5. loaded through NativeRuntime; when a CUDA device is present, a
     differential gate against PyTorch on a bounded set of batch sizes
     (the reference's _verify_rebuilt_artifact, compiler.py:222-272)
  6. manifest written next to the artifact

Arguments that only shape the reference's CPU loop nests keep their meaning
where it exists on the GPU: ``kernel_variant`` fixes the accumulation order
of fused Linear+ReLU (``fused_ikj`` / ``loop_ikj``: the accumulator starts at
the bias, as in src/codegen.cpp:381-396; every other variant adds the bias
after the sum), which the ``simt_exact`` kernel policy reproduces bit for bit.
``gpu_kernel`` (an addition) picks the GPU kernel family.
"""

from __future__ import annotations

import hashlib
import json
import operator
import os
import platform
import sys
from typing import Any, Dict, List, Optional, Sequence, Tuple, Union

import numpy as np
import torch

from . import _native
from .build_native import LIB_PATH
from .emit import compile_shim, emit_source
from .errors import CorrectnessError, InvalidShapeError
from .frontend import IRGraph, export_to_ir
from .graph_blob import POLICIES, blob_sha256, serialize, with_tuning
from .runtime import NativeRuntime

VALID_VARIANTS = ("naive_ijk", "loop_ikj", "tiled", "fused_ikj", "fused_tiled")
GPU_KERNELS = tuple(POLICIES)
ATOL = 1e-4
RTOL = 1e-4


def _sha_file(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def engine_fingerprint() -> str:
    """SHA-256 over the engine library and this package's sources (artifact cache key)."""
    h = hashlib.sha256()
    pkg = os.path.dirname(os.path.abspath(__file__))
    files = [LIB_PATH] + sorted(os.path.join(pkg, f) for f in os.listdir(pkg) if f.endswith(".py"))
    for p in files:
        if os.path.isfile(p):
            h.update(os.path.basename(p).encode())
            h.update(_sha_file(p).encode())
    return h.hexdigest()


def bounded_test_batches(input_shape: Sequence[int], max_batch_size: int, example_batch: int = 1,
                         max_single_batch_bytes: int = 32 << 20) -> List[int]:
    """Batch sizes the differential gate checks: {1, example, 16, cap}, memory-bounded
    (the reference's get_bounded_test_batches, compiler.py:71-113)."""
    if len(input_shape) > 0 and input_shape[0] != -1:
        return [int(input_shape[0])]
    per = max(1, int(np.prod(input_shape[1:])) * 4)
    if per > max_single_batch_bytes:
        raise InvalidShapeError("one sample (%d bytes) exceeds the verification budget" % per)
    cap = min(max_batch_size, 256, max(1, max_single_batch_bytes // per))
    ex = min(max(1, example_batch), cap)
    out = {1, ex, min(16, max_batch_size), cap}
    if max_batch_size * per <= max_single_batch_bytes and max_batch_size <= 256:
        out.add(max_batch_size)
    return sorted(b for b in out if 1 <= b <= cap)


class CompiledModel:
    """A compiled model: runs through the per-model library's C ABI on the GPU."""

    def __init__(self, runtime: NativeRuntime, manifest_data: Dict[str, Any], source: str,
                 opt_report: Dict[str, Any]):
        self._runtime = runtime
        self._manifest = manifest_data
        self._source = source
        self._opt_report = opt_report

    def run(self, input_tensor: Union[np.ndarray, torch.Tensor], batch_size: Optional[int] = None) -> np.ndarray:
        if isinstance(input_tensor, torch.Tensor):
            if input_tensor.is_complex() or not input_tensor.is_floating_point():
                raise TypeError("Unsupported input tensor dtype '%s': ForgeTune requires real numeric float32 input."
                                % input_tensor.dtype)
            if input_tensor.dtype != torch.float32:
                raise TypeError("Unsupported input tensor dtype '%s': ForgeTune requires float32 input "
                                "(no silent casting from '%s')." % (input_tensor.dtype, input_tensor.dtype))
            arr = input_tensor.detach().cpu().numpy()
        else:
            arr = np.asarray(input_tensor)
            if np.iscomplexobj(arr) or arr.dtype != np.float32:
                raise TypeError("Unsupported input tensor dtype '%s': ForgeTune requires float32 input "
                                "(no silent casting from '%s')." % (arr.dtype, arr.dtype))
        return self._runtime.run(arr, batch_size=batch_size)

    __call__ = run

    def run_device(self, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Run on a CUDA tensor; returns (or fills) a CUDA tensor on the current torch stream."""
        if not (isinstance(x, torch.Tensor) and x.is_cuda and x.dtype == torch.float32):
            raise TypeError("run_device needs a float32 CUDA tensor")
        x = x.contiguous()
        b = x.shape[0] if self._runtime.is_dynamic else None
        tail = self._runtime._output_shape_tail
        shape = ((b,) + tuple(tail)) if self._runtime.is_output_dynamic else tuple(self._runtime.expected_output_shape)
        if out is None:
            out = torch.empty(shape, dtype=torch.float32, device=x.device)
        stream = torch.cuda.current_stream(x.device).cuda_stream
        self._runtime.run_device(x.data_ptr(), out.data_ptr(), b or self._runtime.expected_input_shape[0], stream)
        return out

    def optimization_report(self) -> Dict[str, Any]:
        return self._opt_report

    def manifest(self) -> Dict[str, Any]:
        return self._manifest

    def source_code(self) -> str:
        return self._source

    def plan(self) -> Dict[str, Any]:
        """The engine's fused graph, arena plan and launch list."""
        return self._runtime.describe()

    def _dummy(self, batch_size):
        rt = self._runtime
        if rt.is_dynamic:
            b = 1 if batch_size is None else _checked_batch(batch_size, rt.max_batch_size)
            return np.ones((b,) + tuple(rt.expected_input_shape[1:]), np.float32)
        if batch_size is not None and int(batch_size) != rt.expected_input_shape[0]:
            raise InvalidShapeError("Batch size %s does not match static model batch dimension %d"
                                    % (batch_size, rt.expected_input_shape[0]))
        return np.ones(rt.expected_input_shape, np.float32)

    def benchmark(self, warmup_iters: int = 10, measure_iters: int = 50,
                  batch_size: Optional[int] = None) -> Dict[str, Any]:
        """Host-to-host latency statistics of ``run`` (perf_counter_ns)."""
        from .benchmark import benchmark_function
        for name, v, lo in (("warmup_iters", warmup_iters, 0), ("measure_iters", measure_iters, 1)):
            if isinstance(v, bool) or not isinstance(v, int) or v < lo:
                raise TypeError("%s must be an integer >= %d, got %r" % (name, lo, v))
        x = self._dummy(batch_size)
        return benchmark_function(lambda: self._runtime.run(x), warmup_iters, measure_iters)

    def benchmark_kernel(self, iters: int = 1000, batch_size: Optional[int] = None) -> float:
        """Device time per forward pass in microseconds (CUDA events, graph replay)."""
        if isinstance(iters, bool) or not isinstance(iters, int) or iters < 1:
            raise TypeError("iters must be a positive integer >= 1, got %r" % (iters,))
        return self._runtime.benchmark_kernel(self._dummy(batch_size), iters)

    def get_arena_alloc_count(self) -> int:
        return self._runtime.get_arena_alloc_count()

    def get_arena_payload_alloc_count(self) -> int:
        return self._runtime.get_arena_payload_alloc_count()

    def get_arena_block_insertion_count(self) -> int:
        return self._runtime.get_arena_block_insertion_count()

    def reset_arena_alloc_count(self) -> None:
        self._runtime.reset_arena_alloc_count()

    def inject_test_arena_alloc(self) -> None:
        self._runtime.inject_test_arena_alloc()

    def close(self) -> None:
        if self._runtime is not None:
            self._runtime.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def _checked_batch(b, max_b) -> int:
    if isinstance(b, bool):
        raise TypeError("batch_size must be a non-boolean integer, got %r (bool)" % (b,))
    try:
        b = operator.index(b)
    except (TypeError, ValueError):
        raise TypeError("batch_size must be a positive integer, got %r" % (b,))
    if not 1 <= b <= max_b:
        raise InvalidShapeError("Dynamic batch size %d out of valid range [1, %d]" % (b, max_b))
    return b


def _verify(rt: NativeRuntime, oracle, example: np.ndarray, dynamic: bool, max_batch: int) -> Dict[str, Any]:
    """Differential gate against PyTorch (compiler.py:222-272 of the reference)."""
    report = {"batches": [], "max_abs_diff": 0.0}
    batches = bounded_test_batches(rt.expected_input_shape, max_batch, example.shape[0]) if dynamic \
        else [example.shape[0]]
    rng = np.random.default_rng(0)
    for b in batches:
        x = example if b == example.shape[0] else \
            rng.standard_normal((b,) + tuple(example.shape[1:])).astype(np.float32)
        got = rt.run(x)
        want = oracle(x)
        diff = float(np.max(np.abs(got - want))) if got.size else 0.0
        report["batches"].append(b)
        report["max_abs_diff"] = max(report["max_abs_diff"], diff)
        if not np.allclose(got, want, atol=ATOL, rtol=RTOL):
            rel = float(np.max(np.abs(got - want) / np.maximum(np.abs(want), 1e-12)))
            raise CorrectnessError("compiled model differs from PyTorch at batch %d (max abs %.3g)" % (b, diff),
                                   max_abs_diff=diff, max_rel_diff=rel)
    return report


def _module_oracle(model: torch.nn.Module):
    def oracle(x: np.ndarray) -> np.ndarray:
        with torch.no_grad():
            y = model(torch.from_numpy(np.ascontiguousarray(x)))
            if isinstance(y, tuple):
                y = y[0]
            return y.detach().float().numpy()
    return oracle


def _compile_ir(ir: IRGraph, oracle, ex: np.ndarray, output_dir: str, model_name: str, autotune: bool,
                max_autotune_budget: int, opt: str, variant: str, enable_fusion: bool,
                tile_sizes: Optional[Tuple[int, int, int]], max_workspace_bytes: int,
                tuning_batch_sizes: Optional[List[int]], policy: str, devices: Optional[Sequence[int]],
                verify: bool) -> CompiledModel:
    """IR -> graph blob (autotuned on the GPU when asked) -> per-model library
    -> runtime, with the correctness gate against ``oracle``."""
    os.makedirs(output_dir, exist_ok=True)
    max_batch_size = ir.max_batch_size
    bias_first = variant in ("fused_ikj", "loop_ikj")
    blob = serialize(ir, enable_fusion=enable_fusion, bias_first_fused=bias_first, kernel_policy=policy)
    desc = _native.describe_blob(blob)
    if desc["arena_bytes"] > max_workspace_bytes:
        raise ValueError("Configured max_batch_size=%d requires workspace (%d bytes arena) exceeding workspace "
                         "budget %d bytes" % (max_batch_size, desc["arena_bytes"], max_workspace_bytes))

    tuning: Dict[str, Any] = {"status": "off"}
    if autotune:
        if policy == "simt_exact":
            tuning = {"status": "skipped", "reason": "gpu_kernel 'simt_exact' has one kernel per step"}
        elif _native.device_count() == 0:
            tuning = {"status": "skipped", "reason": "no CUDA device visible: the engine's shape rules apply"}
        else:
            from .autotuner import Autotuner
            tuner = Autotuner(atol=ATOL, rtol=RTOL, device=(list(devices)[0] if devices else 0))
            tin_shape = ((-1,) if ir.dynamic else (ex.shape[0],)) + tuple(ex.shape[1:])
            table, treport = tuner.tune(blob, oracle, ex, tin_shape, output_dir, max_budget=max_autotune_budget,
                                        enable_fusion=enable_fusion, tuning_batch_sizes=tuning_batch_sizes)
            blob = with_tuning(blob, table)
            tuning = {"status": "tuned", "cache_hit": treport.get("cache_hit", False), "table": table,
                      "measured_speedup": treport.get("measured_speedup"),
                      "report": os.path.join(os.path.abspath(output_dir), "autotuning_report.json")}
    gsha = blob_sha256(blob)
    cand = {"variant": variant, "gpu_kernel": policy, "enable_fusion": enable_fusion, "opt_level": opt,
            "tile_sizes": list(tile_sizes) if tile_sizes else None}
    prov = hashlib.sha256(json.dumps({"graph": gsha, "cand": cand, "engine": engine_fingerprint()},
                                     sort_keys=True).encode()).hexdigest()[:12]
    cand_dir = os.path.abspath(os.path.join(output_dir, "%s_%s" % (variant, prov)))
    os.makedirs(cand_dir, exist_ok=True)
    blob_path = os.path.join(cand_dir, "graph.ftb")
    cpp_path = os.path.join(cand_dir, "model.cpp")
    so_path = os.path.join(cand_dir, "kernel_%s.so" % prov)
    if not os.path.isfile(so_path):
        with open(blob_path + ".tmp", "wb") as f:
            f.write(blob)
        os.replace(blob_path + ".tmp", blob_path)
        src = emit_source(blob_path, len(blob), gsha, ir.dynamic, desc["max_batch"])
        with open(cpp_path, "w") as f:
            f.write(src)
        compile_shim(cpp_path, so_path, opt)
    with open(cpp_path) as f:
        source = f.read()

    out_node = ir.nodes[ir.output_id]
    if ir.dynamic:
        in_shape = (-1,) + tuple(ex.shape[1:])
        out_shape = tuple(-1 if (i == 0 and out_node.shape[0] == -1) else s for i, s in enumerate(out_node.shape))
    else:
        in_shape = tuple(ex.shape)
        out_shape = tuple(out_node.shape)
    rt = NativeRuntime(so_path, in_shape, out_shape)
    if devices:
        rt.set_devices(list(devices))

    verification: Dict[str, Any] = {"status": "skipped", "reason": "verify=False"}
    if verify:
        if _native.device_count() > 0:
            verification = _verify(rt, oracle, ex, ir.dynamic, desc["max_batch"])
            verification["status"] = "passed"
        else:
            verification = {"status": "skipped", "reason": "no CUDA device visible"}
    report = {"selected_candidate": cand, "plan": {k: desc[k] for k in (
        "arena_bytes", "naive_bytes", "peak_live_bytes", "savings_percent")}, "verification": verification}
    report["autotune"] = tuning
    manifest = {
        "model_name": model_name,
        "input_shape": list(in_shape),
        "output_shape": list(out_shape),
        "kernel_config": cand,
        "artifacts": {"shared_library": so_path, "graph_blob": blob_path, "source": cpp_path,
                      "so_sha256": _sha_file(so_path), "graph_sha256": gsha},
        "graph_hash": gsha,
        "provenance_hash": prov,
        "engine_fingerprint": engine_fingerprint(),
        "platform": sys.platform,
        "machine": platform.machine(),
        "optimization_summary": report,
    }
    tmp = os.path.join(output_dir, "manifest.json.tmp")
    with open(tmp, "w") as f:
        json.dump(manifest, f, indent=2)
    os.replace(tmp, os.path.join(output_dir, "manifest.json"))
    return CompiledModel(rt, manifest, source, report)


def _check_options(autotune, max_autotune_budget, compiler_opt_level, kernel_variant, enable_fusion, tile_sizes,
                   dynamic_batch, max_batch_size, max_workspace_bytes, gpu_kernel) -> Tuple[str, str, str]:
    """The reference compile_model's argument checks (compiler.py:440-520);
    returns (opt level, kernel variant, gpu kernel policy)."""
    if type(max_autotune_budget) is not int or not 1 <= max_autotune_budget <= 8:
        raise ValueError("max_autotune_budget must be an integer between 1 and 8, got %r" % (max_autotune_budget,))
    if type(max_batch_size) is not int or not 1 <= max_batch_size <= 1_000_000:
        raise ValueError("max_batch_size must be an integer between 1 and 1000000, got %r" % (max_batch_size,))
    if dynamic_batch and max_batch_size < 2:
        raise ValueError("Dynamic batch execution requires max_batch_size >= 2 (got max_batch_size=%d). For static "
                         "single-batch execution, set dynamic_batch=False." % max_batch_size)
    if type(max_workspace_bytes) is not int or max_workspace_bytes <= 0:
        raise ValueError("max_workspace_bytes must be a strictly positive integer, got %r" % (max_workspace_bytes,))
    for name, v in (("autotune", autotune), ("dynamic_batch", dynamic_batch), ("enable_fusion", enable_fusion)):
        if type(v) is not bool:
            raise ValueError("%s must be a bool, got %s" % (name, type(v).__name__))
    if not isinstance(compiler_opt_level, str):
        raise TypeError("compiler_opt_level must be a string, got %s" % type(compiler_opt_level).__name__)
    opt = compiler_opt_level if compiler_opt_level.startswith("-") else "-" + compiler_opt_level
    if opt not in ("-O0", "-O1", "-O2", "-O3", "-Os", "-Oz"):
        raise ValueError("Unsupported compiler optimization level: '%s'" % compiler_opt_level)
    if tile_sizes is not None and (not isinstance(tile_sizes, (tuple, list)) or len(tile_sizes) != 3
                                   or any(type(t) is not int or t <= 0 for t in tile_sizes)):
        raise ValueError("tile_sizes must be a 3-tuple/list of positive integers, got %r" % (tile_sizes,))
    if autotune:
        if kernel_variant is not None:
            raise ValueError("Cannot specify 'kernel_variant' ('%s') when autotune=True." % kernel_variant)
        if tile_sizes is not None:
            raise ValueError("Cannot specify 'tile_sizes' (%s) when autotune=True." % (tile_sizes,))
        if opt != "-O2":
            raise ValueError("Cannot override 'compiler_opt_level' when autotune=True.")
    variant = kernel_variant or ("fused_ikj" if (autotune and enable_fusion) else "naive_ijk")
    if variant not in VALID_VARIANTS:
        raise ValueError("Unknown kernel variant: '%s'. Valid variants: %s" % (variant, sorted(VALID_VARIANTS)))
    if not enable_fusion and variant.startswith("fused"):
        raise ValueError("Contradictory options: fused kernel_variant '%s' requested with enable_fusion=False"
                         % variant)
    policy = gpu_kernel or "auto"
    if policy not in GPU_KERNELS:
        raise ValueError("Unknown gpu_kernel '%s'. Valid: %s" % (policy, list(GPU_KERNELS)))
    return opt, variant, policy


def compile_model(model: torch.nn.Module, example_inputs: Tuple[torch.Tensor, ...],
                  output_dir: str = "build/artifacts/model", autotune: bool = True, max_autotune_budget: int = 8,
                  compiler_opt_level: str = "-O2", kernel_variant: Optional[str] = None,
                  enable_fusion: bool = False, tile_sizes: Optional[Tuple[int, int, int]] = None,
                  dynamic_batch: bool = False, max_batch_size: int = 128,
                  max_workspace_bytes: int = 512 * 1024 * 1024, tuning_batch_sizes: Optional[List[int]] = None,
                  gpu_kernel: Optional[str] = None, devices: Optional[Sequence[int]] = None,
                  verify: bool = True) -> CompiledModel:
    """Compile ``model`` into a GPU-backed shared library with the reference C ABI.

    Arguments and checks follow the reference's ``compile_model``.  Additions:
    ``gpu_kernel`` ('auto', 'simt', 'simt_exact', 'tcgen05'; default 'auto'),
    ``devices`` (CUDA device ids to shard the batch over) and ``verify``
    (run the differential gate when a CUDA device is present).
    """
    opt, variant, policy = _check_options(autotune, max_autotune_budget, compiler_opt_level, kernel_variant,
                                          enable_fusion, tile_sizes, dynamic_batch, max_batch_size,
                                          max_workspace_bytes, gpu_kernel)
    for name, p in model.named_parameters():
        if p.device.type != "cpu":
            raise ValueError("Model parameter '%s' is on device '%s'; compile from CPU parameters." % (name, p.device))
    for i, t in enumerate(example_inputs):
        if not isinstance(t, torch.Tensor) or t.device.type != "cpu":
            raise ValueError("Example input %d must be a CPU tensor." % i)

    modes = {n: m.training for n, m in model.named_modules()}
    try:
        model.eval()
        ir: IRGraph = export_to_ir(model, example_inputs, dynamic_batch=dynamic_batch, max_batch_size=max_batch_size)
        oracle = _module_oracle(model)
        ex = example_inputs[0].detach().cpu().float().numpy()
        return _compile_ir(ir, oracle, ex, output_dir, type(model).__name__, autotune, max_autotune_budget, opt,
                           variant, enable_fusion, tile_sizes, max_workspace_bytes, tuning_batch_sizes, policy,
                           devices, verify)
    finally:
        for n, m in model.named_modules():
            if n in modes:
                m.training = modes[n]


def compile_graph_json(graph_json, output_dir: str = "build/artifacts/graph", example_input: Optional[np.ndarray] = None,
                       autotune: bool = True, max_autotune_budget: int = 8, compiler_opt_level: str = "-O2",
                       kernel_variant: Optional[str] = None, enable_fusion: bool = False,
                       tile_sizes: Optional[Tuple[int, int, int]] = None,
                       max_workspace_bytes: int = 512 * 1024 * 1024, tuning_batch_sizes: Optional[List[int]] = None,
                       gpu_kernel: Optional[str] = None, devices: Optional[Sequence[int]] = None,
                       verify: bool = True) -> CompiledModel:
    """Compile a reference ``graph.json`` (schema 2.0: a path, the text or the
    parsed dict, as the reference frontend or CLI writes it) like
    ``compile_model``.  The batch mode and max_batch_size come from the graph;
    the correctness gate and the autotuner compare with a float64 NumPy
    evaluation of the graph (``ir_json.evaluate``).  ``example_input``
    defaults to two rows (or the static batch) of seeded normal values."""
    from .ir_json import evaluate, load_graph_json
    ir = load_graph_json(graph_json)
    opt, variant, policy = _check_options(autotune, max_autotune_budget, compiler_opt_level, kernel_variant,
                                          enable_fusion, tile_sizes, ir.dynamic, ir.max_batch_size,
                                          max_workspace_bytes, gpu_kernel)
    in_shape = ir.nodes[ir.input_id].shape
    if example_input is None:
        rows = min(2, ir.max_batch_size) if ir.dynamic else in_shape[0]
        example_input = np.random.default_rng(1).standard_normal((rows,) + tuple(in_shape[1:])).astype(np.float32)
    ex = np.ascontiguousarray(example_input, dtype=np.float32)
    if tuple(ex.shape[1:]) != tuple(in_shape[1:]) or (not ir.dynamic and ex.shape[0] != in_shape[0]):
        raise InvalidShapeError("example input shape %s does not match the graph input %s" % (ex.shape, in_shape))
    return _compile_ir(ir, lambda x: evaluate(ir, x), ex, output_dir, "graph_json", autotune, max_autotune_budget,
                       opt, variant, enable_fusion, tile_sizes, max_workspace_bytes, tuning_batch_sizes, policy,
                       devices, verify)
