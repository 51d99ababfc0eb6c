"""On-device autotuner: a correctness-gated, timing-driven choice of the GEMM
kernel for every launch-list step and batch range.

It follows the reference's ``Autotuner`` (python/forgetune/autotuner.py): a
bounded, deterministic candidate space with the baseline first
(``get_candidate_space``, :90-127), a correctness gate of every candidate on
the reference's bounded test batches and input kinds (:599-650), interleaved
timing rounds in a shuffled order (:660-700), selection by an improvement of
at least 5 % over the baseline, a 5 % tie band broken by simplicity, and a
degradation safeguard (``select_best_candidate``, :170-290), and a cache
keyed by the graph, the options and the machine (``_compute_cache_key``,
:133-168).

What a candidate is differs.  The reference compiles C++ loop variants and
picks one for the whole model.  Here every candidate is a kernel choice of
the engine -- its shape rules, SIMT FFMA, split-K, or tensor cores with a
tile width, k-block, one SM or an SM pair, and whether a small head is fused
-- applied to every GEMM step.  One profiled forward pass times every step
at once (CUDA events between steps), so the choice is made per step (a fused
head counts with the GEMM that absorbs it) and per batch range, and the
result is a tuning table that the graph blob carries into the compiled
model.  The machine part of the cache key is the GPU: name, compute
capability, SM count, driver and runtime versions.
"""

from __future__ import annotations

import hashlib
import json
import math
import os
from typing import Any, Callable, Dict, List, Optional, Sequence, Tuple

import numpy as np

from . import _native
from .benchmark import get_machine_metadata
from .errors import AutotuningError, CorrectnessError
from .graph_blob import blob_sha256, with_tuning

FAMILY_HEURISTIC, FAMILY_SIMT, FAMILY_SPLITK, FAMILY_TCGEN05 = 0, 1, 2, 3
_FAMILY_NAMES = {0: "shape rules", 1: "simt", 2: "split-k", 3: "tcgen05"}
_STEP_GEMM = 0


class GpuCandidate:
    """One kernel choice, applied to every GEMM step while it is evaluated."""

    def __init__(self, candidate_id: str, family: int, tc_bn: int = 0, tc_bk: int = 0, tc_mh: int = 0,
                 tc_pair: int = 0, fuse_head: bool = True, simplicity: int = 0):
        if not isinstance(candidate_id, str):
            raise TypeError("candidate_id must be a str, got %s" % type(candidate_id).__name__)
        if family not in _FAMILY_NAMES:
            raise ValueError("unknown kernel family %r" % (family,))
        if type(fuse_head) is not bool:
            raise TypeError("fuse_head must be a bool, got %s" % type(fuse_head).__name__)
        self.candidate_id = candidate_id
        self.family = family
        self.tc_bn, self.tc_bk, self.tc_mh, self.tc_pair = tc_bn, tc_bk, tc_mh, tc_pair
        self.fuse_head = fuse_head
        self.simplicity = simplicity  # lower is simpler: the tie-break

    @property
    def enable_fusion(self) -> bool:
        return self.fuse_head

    def record(self, step: int, lo: int, hi: int) -> List[int]:
        return [step, lo, hi, self.family, self.tc_bn, self.tc_bk, self.tc_mh, self.tc_pair, int(self.fuse_head)]

    def to_dict(self) -> Dict[str, Any]:
        return {"candidate_id": self.candidate_id, "family": _FAMILY_NAMES[self.family], "tc_bn": self.tc_bn,
                "tc_bk": self.tc_bk, "tc_mh": self.tc_mh, "tc_pair": self.tc_pair, "fuse_head": self.fuse_head,
                "simplicity": self.simplicity}


def _gen_test_cases(rng: np.random.Generator, shape: Tuple[int, ...]):
    """The reference's gate inputs (autotuner.py:620-625): normal, zeros,
    negative, uniform(-5, 5)."""
    yield rng.standard_normal(shape).astype(np.float32)
    yield np.zeros(shape, dtype=np.float32)
    yield -np.abs(rng.standard_normal(shape).astype(np.float32))
    yield rng.uniform(-5.0, 5.0, size=shape).astype(np.float32)


class Autotuner:
    def __init__(self, cache_dir: Optional[str] = None, atol: float = 1e-4, rtol: float = 1e-4, device: int = 0,
                 timing_budget_ms: float = 20.0, device_buffer_budget: int = 2 << 30):
        self.cache_dir = cache_dir or os.path.join(os.getcwd(), "build", "tuning_cache")
        self.atol = atol
        self.rtol = rtol
        self.device = device
        self.timing_budget_ms = timing_budget_ms
        self.device_buffer_budget = device_buffer_budget

    # ------------------------------------------------------------------ space
    def get_candidate_space(self, max_budget: int = 8, force_fusion: bool = False,
                            enable_fusion: Optional[bool] = None) -> List[GpuCandidate]:
        """Bounded, deterministic candidates, the baseline (the engine's shape
        rules) first.  enable_fusion=False: no candidate fuses a head (each is
        turned into its non-fusing form, duplicates dropped); force_fusion:
        only candidates that fuse."""
        if type(max_budget) is not int or isinstance(max_budget, bool) or not 1 <= max_budget <= 8:
            raise ValueError("max_budget must be an integer between 1 and 8, got %r (%s)"
                             % (max_budget, type(max_budget).__name__))
        if enable_fusion is False and force_fusion:
            raise ValueError("Contradictory autotuner options: enable_fusion cannot be False when force_fusion is True")
        cands = [
            GpuCandidate("engine_default", FAMILY_HEURISTIC, simplicity=0),
            GpuCandidate("tc_pair_k16", FAMILY_TCGEN05, 0, 16, 0, 2, simplicity=2),
            GpuCandidate("tc_sm_k16", FAMILY_TCGEN05, 0, 16, 1, 1, simplicity=1),
            GpuCandidate("simt_ffma", FAMILY_SIMT, simplicity=1),
            GpuCandidate("split_k", FAMILY_SPLITK, simplicity=1),
            GpuCandidate("tc_pair_k32", FAMILY_TCGEN05, 0, 32, 0, 2, simplicity=3),
            GpuCandidate("tc_sm_n128_k16", FAMILY_TCGEN05, 128, 16, 1, 1, simplicity=2),
            GpuCandidate("tc_pair_k16_head_apart", FAMILY_TCGEN05, 0, 16, 0, 2, fuse_head=False, simplicity=3),
        ]
        if enable_fusion is False:
            seen, out = set(), []
            for c in cands:
                c = GpuCandidate(c.candidate_id, c.family, c.tc_bn, c.tc_bk, c.tc_mh, c.tc_pair, False, c.simplicity)
                key = (c.family, c.tc_bn, c.tc_bk, c.tc_mh, c.tc_pair)
                if key not in seen:
                    seen.add(key)
                    out.append(c)
            cands = out
        elif force_fusion:
            cands = [c for c in cands if c.fuse_head]
        return cands[:max_budget]

    # ---------------------------------------------------------------- batches
    def timing_batches(self, dynamic: bool, max_batch: int, static_batch: int, in_elems: int, out_elems: int,
                       tuning_batch_sizes: Optional[Sequence[int]] = None) -> List[int]:
        """Batch sizes timed: the caller's list, else 1, 16, 256, 4096, 65536
        and max_batch (up to max_batch and the device-buffer budget)."""
        if not dynamic:
            return [static_batch]
        if tuning_batch_sizes is not None:
            if not isinstance(tuning_batch_sizes, (list, tuple)) or not tuning_batch_sizes:
                raise ValueError("tuning_batch_sizes must be a non-empty list of positive integers")
            for b in tuning_batch_sizes:
                if type(b) is bool or type(b) is not int or b <= 0:
                    raise ValueError("Invalid tuning batch size: %r" % (b,))
                if b > max_batch:
                    raise ValueError("tuning batch size %d exceeds max_batch_size %d" % (b, max_batch))
            out = sorted(set(tuning_batch_sizes))
        else:
            out = sorted({b for b in (1, 16, 256, 4096, 65536, max_batch) if b <= max_batch})
        per = max(1, (in_elems + out_elems) * 4)
        cap = max(1, self.device_buffer_budget // per)
        kept = [b for b in out if b <= cap]
        return kept or [min(out[0], cap)]

    @staticmethod
    def buckets(batches: Sequence[int], max_batch: int) -> List[Tuple[int, int]]:
        """Batch ranges, one per timed batch size, split at geometric midpoints."""
        bs = sorted(batches)
        out = []
        lo = 1
        for i, b in enumerate(bs):
            hi = max_batch if i + 1 == len(bs) else max(b, int(math.floor(math.sqrt(b * bs[i + 1]))))
            out.append((lo, hi))
            lo = hi + 1
        return out

    # ------------------------------------------------------------------ cache
    def _compute_cache_key(self, blob: bytes, input_shape: Tuple[int, ...], max_budget: int, force_fusion: bool,
                           enable_fusion: Optional[bool], tuning_batch_sizes: Optional[Sequence[int]],
                           device_info: Dict[str, Any], candidates: List[GpuCandidate]) -> str:
        from .compiler import engine_fingerprint
        h = hashlib.sha256()
        h.update(b"forgetune_b200_gpu_tuning_1_")
        h.update(blob_sha256(with_tuning(blob, [])).encode())
        for part in (input_shape, max_budget, force_fusion, enable_fusion, tuning_batch_sizes,
                     "atol_%.1e_rtol_%.1e" % (self.atol, self.rtol), engine_fingerprint(),
                     json.dumps(device_info, sort_keys=True),
                     json.dumps([c.to_dict() for c in candidates], sort_keys=True)):
            h.update(str(part).encode())
        return h.hexdigest()

    # -------------------------------------------------------------- selection
    def select(self, unit_costs: Dict[str, float], cands: Dict[str, GpuCandidate],
               base_id: str) -> Tuple[str, str]:
        """The reference's rule on one unit (a GEMM step, with the head it may
        absorb) in one batch range: keep the baseline unless a candidate is
        at least 5 % faster; among those within 5 % of the fastest, take the
        simplest.  Returns (candidate id, rationale)."""
        base = unit_costs.get(base_id)
        if base is None or base <= 0:
            return base_id, "baseline not timed"
        improving = [(cid, t) for cid, t in unit_costs.items() if t > 0 and base / t >= 1.05]
        if not improving:
            return base_id, "no candidate at least 5% faster than the baseline; baseline kept"
        fastest = min(t for _, t in improving)
        tier = [(cid, t) for cid, t in improving if t <= fastest * 1.05]
        tier.sort(key=lambda x: (cands[x[0]].simplicity, x[1]))
        cid, t = tier[0]
        return cid, "%s: %.2fx faster than the baseline (%.1f us vs %.1f us)" % (cid, base / t, t * 1e3, base * 1e3)

    # ------------------------------------------------------------------- tune
    def tune(self, blob: bytes, oracle: Callable[[np.ndarray], np.ndarray], example_input: np.ndarray,
             input_shape: Tuple[int, ...], artifacts_dir: str, max_budget: int = 8, use_cache: bool = True,
             force_fusion: bool = False, enable_fusion: Optional[bool] = None,
             tuning_batch_sizes: Optional[List[int]] = None) -> Tuple[List[List[int]], Dict[str, Any]]:
        """Tune the graph in ``blob`` on this process's CUDA device ``device``.

        ``oracle`` maps an input batch to the expected output (the PyTorch
        model); ``input_shape`` has -1 for a dynamic batch.  Returns the
        tuning table (records for ``graph_blob.with_tuning``) and the report,
        also written to ``artifacts_dir/autotuning_report.json``."""
        import torch  # device buffers for the timing runs

        if type(max_budget) is not int or isinstance(max_budget, bool) or not 1 <= max_budget <= 8:
            raise ValueError("max_budget must be an integer between 1 and 8, got %r" % (max_budget,))
        if type(force_fusion) is not bool:
            raise TypeError("force_fusion must be a bool, got %r" % (force_fusion,))
        if enable_fusion is not None and type(enable_fusion) is not bool:
            raise TypeError("enable_fusion must be a bool or None, got %r" % (enable_fusion,))
        if _native.device_count() <= self.device:
            raise AutotuningError("no CUDA device %d to tune on" % self.device)
        os.makedirs(artifacts_dir, exist_ok=True)
        blob = with_tuning(blob, [])
        info = _native.device_info(self.device)
        cands = self.get_candidate_space(max_budget, force_fusion=force_fusion, enable_fusion=enable_fusion)
        by_id = {c.candidate_id: c for c in cands}
        base_id = cands[0].candidate_id
        key = self._compute_cache_key(blob, tuple(input_shape), max_budget, force_fusion, enable_fusion,
                                      tuning_batch_sizes, info, cands)
        cache_file = os.path.join(self.cache_dir, key + ".json")
        report_path = os.path.join(artifacts_dir, "autotuning_report.json")
        if use_cache and os.path.isfile(cache_file):
            try:
                with open(cache_file) as f:
                    cached = json.load(f)
                table = cached["selected_table"]
                if not isinstance(table, list) or any(
                        not isinstance(r, list) or len(r) != 9 or any(type(v) is not int for v in r) for r in table):
                    raise ValueError("invalid cached table")
                _native.describe_blob(with_tuning(blob, table))  # the engine accepts it
                cached["cache_hit"] = True
                _write_json(report_path, cached)
                return table, cached
            except Exception:
                pass  # invalid or stale: tune again

        eng = _native.EngineModel(blob)
        try:
            return self._tune_engine(eng, blob, oracle, example_input, input_shape, cands, by_id, base_id, info,
                                     tuning_batch_sizes, key, cache_file, report_path, use_cache, torch)
        finally:
            eng.close()

    def _tune_engine(self, eng, blob, oracle, example_input, input_shape, cands, by_id, base_id, info,
                     tuning_batch_sizes, key, cache_file, report_path, use_cache, torch):
        from .compiler import bounded_test_batches
        desc = eng.desc
        dynamic = bool(desc["dynamic"])
        max_batch = int(desc["max_batch"])
        static_batch = int(desc["static_batch"])
        steps = desc["steps"]
        gemms = [i for i, s in enumerate(steps) if s["kind"] == _STEP_GEMM]
        # a unit: a GEMM step and the steps one launch of it may also compute
        # -- the head it may absorb, or the next layer (and that layer's head)
        # of a two-layer kernel -- so that every candidate's cost covers the
        # same work
        units = []
        for i in gemms:
            st = steps[i]
            if st["head_of"] >= 0 or st.get("mlp_of", -1) >= 0:
                continue
            unit = [i]
            if st.get("mlp_step", -1) >= 0:
                j = st["mlp_step"]
                unit.append(j)
                if steps[j]["head_step"] >= 0:
                    unit.append(steps[j]["head_step"])
            elif st["head_step"] >= 0:
                unit.append(st["head_step"])
            units.append(unit)
        eng.set_devices([self.device])
        eng.prepare()

        def forced(c: GpuCandidate) -> List[List[int]]:
            if c.family == FAMILY_HEURISTIC and c.fuse_head:
                return []
            lo, hi = (1, max_batch) if dynamic else (static_batch, static_batch)
            return [c.record(s, lo, hi) for s in gemms]

        # ---- phase 1: correctness gate -------------------------------------
        test_batches = bounded_test_batches(tuple(input_shape), max_batch, example_input.shape[0]) if dynamic \
            else [static_batch]
        expected_example = oracle(example_input)
        evaluations: List[Dict[str, Any]] = []
        passed: List[GpuCandidate] = []
        for c in cands:
            entry: Dict[str, Any] = {"candidate": c.to_dict(), "status": "pending", "rejection_reason": None}
            try:
                eng.set_tuning(forced(c))
                got = self._run_host(eng, example_input, expected_example.shape)
                if not np.allclose(got, expected_example, atol=self.atol, rtol=self.rtol):
                    raise CorrectnessError("mismatch vs PyTorch on the example input: max_abs=%g"
                                           % float(np.max(np.abs(got - expected_example))))
                rng = np.random.default_rng(42)
                for b in test_batches:
                    for x in _gen_test_cases(rng, (b,) + tuple(example_input.shape[1:])):
                        want = oracle(x)
                        got = self._run_host(eng, x, want.shape)
                        if not np.allclose(got, want, atol=self.atol, rtol=self.rtol):
                            max_abs = float(np.max(np.abs(got - want)))
                            raise CorrectnessError("mismatch vs PyTorch at batch %d: max_abs=%g" % (b, max_abs),
                                                   max_abs_diff=max_abs)
                entry["status"] = "passed"
                passed.append(c)
            except Exception as e:  # rejected, like the reference's gate
                entry["status"] = "correctness_failed"
                entry["rejection_reason"] = "%s: %s" % (type(e).__name__, e)
            evaluations.append(entry)
        if not any(c.candidate_id == base_id for c in passed):
            raise AutotuningError("the baseline candidate failed the correctness gate: %s"
                                  % evaluations[0]["rejection_reason"])

        # ---- phase 2: interleaved timing -----------------------------------
        in_elems, out_elems = int(desc["in_elems"]), int(desc["out_elems"])
        batches = self.timing_batches(dynamic, max_batch, static_batch, in_elems, out_elems, tuning_batch_sizes)
        dev = torch.device("cuda", self.device)
        bmax = max(batches)
        x_dev = torch.empty(max(1, bmax * in_elems if dynamic else in_elems), dtype=torch.float32, device=dev)
        y_dev = torch.empty(max(1, bmax * out_elems if dynamic else out_elems), dtype=torch.float32, device=dev)
        _native.philox_normal(x_dev.data_ptr(), 1, 0, x_dev.numel())
        stream = torch.cuda.current_stream(dev)
        samples = {c.candidate_id: {b: [] for b in batches} for c in passed}  # per-step ms arrays
        orders = []
        for rnd in range(3):
            order = list(passed)
            np.random.default_rng(2000 + rnd).shuffle(order)
            orders.append([c.candidate_id for c in order])
            for c in order:
                eng.set_tuning(forced(c))
                for b in batches:
                    samples[c.candidate_id][b].extend(self._time_steps(eng, x_dev, y_dev, b, dynamic, in_elems,
                                                                       out_elems, stream, torch))
        med = {cid: {b: np.median(np.array(v), axis=0) for b, v in per.items()} for cid, per in samples.items()}
        for entry in evaluations:
            cid = entry["candidate"]["candidate_id"]
            if cid in med:
                entry["per_batch_step_ms"] = {str(b): [round(float(t), 5) for t in med[cid][b]] for b in batches}
                entry["per_batch_forward_ms"] = {str(b): round(float(med[cid][b].sum()), 5) for b in batches}

        # ---- phase 3: per-unit, per-range selection --------------------------
        ranges = self.buckets(batches, max_batch) if dynamic else [(static_batch, static_batch)]
        chosen: Dict[Tuple[int, int], str] = {}  # (unit index, batch index) -> candidate id
        rationale = []
        for bi, b in enumerate(batches):
            for ui, unit in enumerate(units):
                costs = {cid: float(sum(med[cid][b][s] for s in unit)) for cid in med}
                cid, why = self.select(costs, by_id, base_id)
                chosen[(ui, bi)] = cid
                rationale.append({"steps": unit, "batch": b, "batch_range": list(ranges[bi]), "selected": cid,
                                  "rationale": why})
        table = self._table(units, ranges, chosen, by_id, base_id)

        # ---- phase 4: the combined table: gate, then degradation safeguard --
        eng.set_tuning(table)
        got = self._run_host(eng, example_input, expected_example.shape)
        if not np.allclose(got, expected_example, atol=self.atol, rtol=self.rtol):
            raise CorrectnessError("the combined tuning table fails the gate on the example input")
        combined = {b: [] for b in batches}
        base_fw = {b: float(med[base_id][b].sum()) for b in batches}
        for _ in range(3):
            for b in batches:
                combined[b].extend(self._time_steps(eng, x_dev, y_dev, b, dynamic, in_elems, out_elems, stream,
                                                    torch))
        comb_fw = {b: float(np.median(np.array(combined[b]), axis=0).sum()) for b in batches}
        dropped = []
        for bi, b in enumerate(batches):
            if comb_fw[b] >= base_fw[b] and any(chosen[(ui, bi)] != base_id for ui in range(len(units))):
                for ui in range(len(units)):
                    chosen[(ui, bi)] = base_id
                dropped.append(b)
        if dropped:
            table = self._table(units, ranges, chosen, by_id, base_id)
            eng.set_tuning(table)

        report = {
            "schema_version": "2.0-gpu",
            "cache_key": key,
            "selected_table": table,
            "table_fields": ["step", "batch_lo", "batch_hi", "family", "tc_bn", "tc_bk", "tc_mh", "tc_pair",
                             "fuse_head"],
            "selections": rationale,
            "safeguard_reverted_batches": dropped,
            "baseline_candidate": base_id,
            "baseline_forward_ms": {str(b): base_fw[b] for b in batches},
            "tuned_forward_ms": {str(b): (base_fw[b] if b in dropped else comb_fw[b]) for b in batches},
            "measured_speedup": {str(b): base_fw[b] / (base_fw[b] if b in dropped else comb_fw[b])
                                 for b in batches},
            "workload_batch_profile": batches,
            "batch_ranges": [list(r) for r in ranges],
            "correctness_batches": test_batches,
            "round_execution_orders": orders,
            "device": info,
            "machine_metadata": get_machine_metadata(),
            "candidate_evaluations": evaluations,
            "cache_hit": False,
        }
        if use_cache:
            os.makedirs(self.cache_dir, exist_ok=True)
            _write_json(cache_file, report)
        _write_json(report_path, report)
        return table, report

    @staticmethod
    def _table(units, ranges, chosen, by_id, base_id) -> List[List[int]]:
        """Records for every non-baseline choice, adjacent ranges merged."""
        table = []
        for ui, unit in enumerate(units):
            bi = 0
            while bi < len(ranges):
                cid = chosen[(ui, bi)]
                bj = bi
                while bj + 1 < len(ranges) and chosen[(ui, bj + 1)] == cid:
                    bj += 1
                if cid != base_id:
                    c = by_id[cid]
                    for s in unit:
                        table.append(c.record(s, ranges[bi][0], ranges[bj][1]))
                bi = bj + 1
        return table

    @staticmethod
    def _run_host(eng, x: np.ndarray, out_shape) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.empty(out_shape, dtype=np.float32)
        rc = eng.run(x, y)
        if rc != 0:
            raise CorrectnessError("run failed with status %d: %s" % (rc, _native.last_error()))
        return y

    def _time_steps(self, eng, x_dev, y_dev, b, dynamic, in_elems, out_elems, stream, torch) -> List[np.ndarray]:
        """Per-step device times (ms) of a few forward passes at batch b."""
        n_in = b * in_elems if dynamic else in_elems
        n_out = b * out_elems if dynamic else out_elems
        s = stream.cuda_stream
        for slot in range(3):
            eng.run_device_profiled(x_dev.data_ptr(), n_in, y_dev.data_ptr(), n_out, b, s, slot)
        torch.cuda.synchronize()
        first = float(np.sum(eng.profile_read(0)))
        reps = int(min(50, max(5, math.ceil(self.timing_budget_ms / max(first, 1e-3)))))
        for slot in range(reps):
            eng.run_device_profiled(x_dev.data_ptr(), n_in, y_dev.data_ptr(), n_out, b, s, slot)
        torch.cuda.synchronize()
        return [np.array(eng.profile_read(slot)) for slot in range(reps)]


def _write_json(path: str, data: Dict[str, Any]) -> None:
    tmp = path + ".tmp"
    with open(tmp, "w") as f:
        json.dump(data, f, indent=2)
    os.replace(tmp, path)
