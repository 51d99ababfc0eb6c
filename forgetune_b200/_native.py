"""ctypes binding of the engine ABI in libforgetune_b200.so (include/forgetune_b200.h).

There is no fallback: if the library is missing or cannot load, every entry
point raises :class:`ForgeTuneRuntimeError`.
"""

from __future__ import annotations

import ctypes
import json
import os
import threading
from typing import Optional

from .build_native import LIB_PATH
from .errors import ForgeTuneRuntimeError

_lock = threading.Lock()
_lib: Optional[ctypes.CDLL] = None

c_void_p, c_size_t, c_int, c_int64, c_double, c_char_p, c_uint64 = (
    ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_int64, ctypes.c_double, ctypes.c_char_p,
    ctypes.c_uint64)

_SIGS = {
    "ftb_last_error": ([], c_char_p),
    "ftb_describe_blob": ([c_void_p, c_size_t, c_void_p, c_size_t], c_int),
    "ftb_model_create": ([c_void_p, c_size_t, ctypes.POINTER(c_void_p)], c_int),
    "ftb_model_destroy": ([c_void_p], None),
    "ftb_model_set_devices": ([c_void_p, c_void_p, c_int], c_int),
    "ftb_model_set_policy": ([c_void_p, c_int], c_int),
    "ftb_model_prepare": ([c_void_p], c_int),
    "ftb_model_set_step_config": ([c_void_p, c_int, c_int, c_int, c_int, c_int, c_int], c_int),
    "ftb_model_set_fault_injection": ([c_void_p, c_int], c_int),
    "ftb_model_run": ([c_void_p, c_void_p, c_size_t, c_void_p, c_size_t, c_int64, c_int], c_int),
    "ftb_model_run_device": ([c_void_p, c_void_p, c_size_t, c_void_p, c_size_t, c_int64, c_void_p], c_int),
    "ftb_model_run_device_profiled": ([c_void_p, c_void_p, c_size_t, c_void_p, c_size_t, c_int64, c_void_p, c_int],
                                      c_int),
    "ftb_model_profile_read": ([c_void_p, c_int, c_void_p, c_int], c_int),
    "ftb_model_benchmark": ([c_void_p, c_void_p, c_size_t, c_void_p, c_size_t, c_int], c_double),
    "ftb_model_is_dynamic": ([c_void_p], c_int),
    "ftb_model_max_batch": ([c_void_p], c_int64),
    "ftb_model_counter": ([c_void_p, c_int], c_size_t),
    "ftb_model_reset_counters": ([c_void_p], None),
    "ftb_model_inject_alloc": ([c_void_p], None),
    "ftb_model_describe": ([c_void_p, c_void_p, c_size_t], c_int),
    "ftb_device_count": ([], c_int),
    "ftb_device_info": ([c_int, c_void_p, c_size_t], c_int),
    "ftb_model_set_tuning": ([c_void_p, c_void_p, c_int], c_int),
    "ftb_philox_normal": ([c_void_p, c_uint64, c_uint64, c_uint64, c_void_p], c_int),
    "ftb_small_gemm_noalloc": ([c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64,
                                ctypes.c_uint32, c_void_p], c_int),
}

EXPORTED = sorted(_SIGS)


def lib() -> ctypes.CDLL:
    """The loaded engine library (loaded once, RTLD_GLOBAL so model shims share it)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.isfile(LIB_PATH):
                raise ForgeTuneRuntimeError(
                    "libforgetune_b200.so is not built (%s); run `python -m forgetune_b200.build_native`" % LIB_PATH)
            try:
                L = ctypes.CDLL(LIB_PATH, mode=ctypes.RTLD_GLOBAL)
            except OSError as e:
                raise ForgeTuneRuntimeError("cannot load %s: %s" % (LIB_PATH, e)) from e
            for name, (argt, rest) in _SIGS.items():
                fn = getattr(L, name)
                fn.argtypes = argt
                fn.restype = rest
            _lib = L
    return _lib


def last_error() -> str:
    return (lib().ftb_last_error() or b"").decode("utf-8", "replace")


def describe_blob(blob: bytes) -> dict:
    """Fuse + plan a graph blob on the host and return the engine's JSON description."""
    L = lib()
    n = L.ftb_describe_blob(blob, len(blob), None, 0)
    if n < 0:
        raise ForgeTuneRuntimeError("graph rejected by the engine: %s" % last_error())
    buf = ctypes.create_string_buffer(n + 1)
    L.ftb_describe_blob(blob, len(blob), buf, n + 1)
    return json.loads(buf.value.decode())


def device_count() -> int:
    return int(lib().ftb_device_count())


def device_info(device: int = 0) -> dict:
    """Name, compute capability, SM count, memory and driver / runtime versions of a CUDA device."""
    L = lib()
    n = L.ftb_device_info(device, None, 0)
    if n < 0:
        raise ForgeTuneRuntimeError("ftb_device_info failed (%d): %s" % (n, last_error()))
    buf = ctypes.create_string_buffer(n + 1)
    L.ftb_device_info(device, buf, n + 1)
    return json.loads(buf.value.decode())


def philox_normal(ptr: int, seed: int, first: int, count: int, stream: int = 0) -> None:
    rc = lib().ftb_philox_normal(ptr, seed, first, count, stream or None)
    if rc != 0:
        raise ForgeTuneRuntimeError("ftb_philox_normal failed (%d): %s" % (rc, last_error()))


class EngineModel:
    """A model handle of the engine ABI built straight from a graph blob.

    ``CompiledModel`` goes through the per-model library; this class is the
    same engine without the shim, for callers that hold a blob (benchmarks,
    tests, embedding in another host)."""

    def __init__(self, blob: bytes):
        self._blob = bytes(blob)
        h = c_void_p()
        rc = lib().ftb_model_create(self._blob, len(self._blob), ctypes.byref(h))
        if rc != 0:
            raise ForgeTuneRuntimeError("ftb_model_create failed (%d): %s" % (rc, last_error()))
        self.handle = h.value
        self.desc = self.describe()

    def _check(self, rc: int, what: str) -> None:
        if rc != 0:
            raise ForgeTuneRuntimeError("%s failed (%d): %s" % (what, rc, last_error()))

    def describe(self) -> dict:
        n = lib().ftb_model_describe(self.handle, None, 0)
        buf = ctypes.create_string_buffer(n + 1)
        lib().ftb_model_describe(self.handle, buf, n + 1)
        return json.loads(buf.value.decode())

    def set_devices(self, ids) -> None:
        arr = (c_int * max(1, len(ids)))(*ids)
        self._check(lib().ftb_model_set_devices(self.handle, ctypes.cast(arr, c_void_p), len(ids)), "set_devices")

    def set_policy(self, policy: int) -> None:
        self._check(lib().ftb_model_set_policy(self.handle, int(policy)), "set_policy")

    def prepare(self) -> None:
        self._check(lib().ftb_model_prepare(self.handle), "prepare")

    def set_step_config(self, step: int, tc_bn: int = 0, tc_bk: int = 0, tc_mh: int = 0, tc_pair: int = 0,
                        fuse_head: bool = True) -> None:
        self._check(lib().ftb_model_set_step_config(self.handle, step, tc_bn, tc_bk, tc_mh, tc_pair,
                                                    int(fuse_head)), "set_step_config")

    def set_tuning(self, records) -> None:
        """Replace the tuned kernel table: records of 9 ints
        (step, batch_lo, batch_hi, family, tc_bn, tc_bk, tc_mh, tc_pair, fuse_head)."""
        flat = [int(v) for r in records for v in r]
        if any(len(r) != 9 for r in records):
            raise ValueError("tuning records have 9 fields")
        arr = (ctypes.c_int64 * max(1, len(flat)))(*flat)
        self._check(lib().ftb_model_set_tuning(self.handle, ctypes.cast(arr, c_void_p), len(records)), "set_tuning")

    def run(self, x, out, api: int = 2) -> int:
        return int(lib().ftb_model_run(self.handle, x.ctypes.data, x.size, out.ctypes.data, out.size,
                                       x.shape[0] if self.desc["dynamic"] else 0, api))

    def run_device(self, d_in: int, in_count: int, d_out: int, out_count: int, batch: int, stream: int = 0) -> None:
        self._check(lib().ftb_model_run_device(self.handle, d_in, in_count, d_out, out_count, batch, stream),
                    "run_device")

    def run_device_profiled(self, d_in: int, in_count: int, d_out: int, out_count: int, batch: int,
                            stream: int, slot: int) -> None:
        self._check(lib().ftb_model_run_device_profiled(self.handle, d_in, in_count, d_out, out_count, batch,
                                                        stream, slot), "run_device_profiled")

    def profile_read(self, slot: int):
        n = len(self.desc["steps"])
        buf = (ctypes.c_float * max(1, n))()
        rc = lib().ftb_model_profile_read(self.handle, slot, ctypes.cast(buf, c_void_p), n)
        if rc < 0:
            self._check(rc, "profile_read")
        return [float(buf[i]) for i in range(n)]

    def graph_kernels(self) -> int:
        """Kernels one replay of the most recently captured launch-list graph launches."""
        return int(lib().ftb_model_counter(self.handle, 4))

    def close(self) -> None:
        if self.handle:
            lib().ftb_model_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
