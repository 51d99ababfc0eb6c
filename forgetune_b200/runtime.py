"""ctypes loader for a compiled model library.

Same interface, argument meaning and errors as the reference's
``NativeRuntime`` (python/forgetune/runtime.py:16-544): it binds
``forgetune_run_v2`` / ``forgetune_run_v1`` / ``forgetune_run`` by probing the
exports, checks dtype, rank, feature dimensions and the batch range before
calling, allocates the output, and maps native status codes to exceptions.
It also binds the additions of this backend (device-pointer run, device
selection, create / destroy, plan description).
"""

from __future__ import annotations

import ctypes
import json
import math
import operator
import os
from typing import Optional, Sequence, Tuple

import numpy as np

from .errors import ForgeTuneRuntimeError, InvalidShapeError

_STATUS = {
    -1: "Null pointer supplied to native kernel",
    -2: "Input element count or batch size mismatch",
    -3: "Output element count mismatch",
    -4: "Native arena allocation failed",
    -5: "CUDA error while running the model",
    -6: "Invalid graph or configuration",
}

_RUN5 = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int64]
_RUN4 = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t]


def _positive_int(v, what: str, exc=TypeError) -> int:
    if isinstance(v, bool):
        raise exc("%s must be a strictly positive non-boolean integer, got %r (bool)" % (what, v))
    try:
        iv = operator.index(v)
    except (TypeError, ValueError):
        raise exc("%s must be a strictly positive non-boolean integer, got %r (%s)" % (what, v, type(v).__name__))
    if iv <= 0:
        raise exc("%s must be a strictly positive non-boolean integer, got %d" % (what, iv))
    return iv


class NativeRuntime:
    def __init__(self, dll_path: str, expected_input_shape: Tuple[int, ...],
                 expected_output_shape: Tuple[int, ...], max_batch_size: Optional[int] = None):
        if max_batch_size is not None:
            max_batch_size = _positive_int(max_batch_size, "max_batch_size")
        self._configured_max_batch_size = max_batch_size
        self.original_dll_path = os.path.abspath(dll_path)
        self.expected_input_shape = tuple(expected_input_shape)
        self.expected_output_shape = tuple(expected_output_shape)
        self.is_closed = False
        self.is_shape_dynamic = len(self.expected_input_shape) > 0 and self.expected_input_shape[0] == -1
        if self.is_shape_dynamic:
            self.total_input_count = self.total_output_count = -1
        else:
            self.total_input_count = int(math.prod(self.expected_input_shape))
            self.total_output_count = int(math.prod(self.expected_output_shape))
        if not os.path.isfile(self.original_dll_path):
            raise FileNotFoundError("Shared library not found: %s" % self.original_dll_path)
        try:
            self.lib = ctypes.CDLL(self.original_dll_path)
        except OSError as e:
            raise OSError("Failed to load shared library '%s': %s" % (self.original_dll_path, e)) from e
        self._bind()

    # ------------------------------------------------------------------ binding
    def _fn(self, name: str, argtypes, restype):
        if not hasattr(self.lib, name):
            return None
        f = getattr(self.lib, name)
        f.argtypes = argtypes
        f.restype = restype
        return f

    def _bind(self) -> None:
        L = self.lib
        if not any(hasattr(L, n) for n in ("forgetune_run_v2", "forgetune_run_v1", "forgetune_run")):
            raise ForgeTuneRuntimeError(
                "Missing exported inference entry point in %s (expected forgetune_run_v2, forgetune_run_v1, "
                "or forgetune_run)" % self.original_dll_path)
        if hasattr(L, "forgetune_is_dynamic"):
            L.forgetune_is_dynamic.restype = ctypes.c_int
            self.is_dynamic = bool(L.forgetune_is_dynamic())
        else:
            self.is_dynamic = hasattr(L, "forgetune_run_v2") or self.is_shape_dynamic
        native_limit = None
        mb = self._fn("forgetune_max_batch", [], ctypes.c_int64)
        if mb is not None:
            native_limit = int(mb())
        if self._configured_max_batch_size is not None:
            if native_limit is not None and self._configured_max_batch_size > native_limit:
                raise ValueError("Configured max_batch_size (%d) exceeds compiled native library maximum (%d)"
                                 % (self._configured_max_batch_size, native_limit))
            self.max_batch_size = self._configured_max_batch_size
        elif native_limit is not None:
            self.max_batch_size = native_limit
        else:
            self.max_batch_size = 128 if self.is_dynamic else (
                self.expected_input_shape[0] if self.expected_input_shape else 1)
        self.is_output_dynamic = len(self.expected_output_shape) > 0 and self.expected_output_shape[0] == -1
        self._output_shape_tail = (tuple(self.expected_output_shape[1:]) if self.is_output_dynamic
                                   else self.expected_output_shape)
        self.run_v2_fn = self._fn("forgetune_run_v2", _RUN5, ctypes.c_int)
        self.run_v1_fn = self._fn("forgetune_run_v1", _RUN4, ctypes.c_int)
        if self.is_dynamic:
            self.run_dynamic_fn = self.run_v2_fn or self._fn("forgetune_run", _RUN5, ctypes.c_int)
            self.run_v1_dynamic_fn = None if self.run_dynamic_fn is not None else self.run_v1_fn
            if self.run_dynamic_fn is None and self.run_v1_dynamic_fn is None:
                raise ForgeTuneRuntimeError("Missing dynamic entry point in %s" % self.original_dll_path)
            self.run_fn = self.run_dynamic_fn or self.run_v1_dynamic_fn
            if self.run_v2_fn is None:
                self.run_v2_fn = self.run_dynamic_fn
        else:
            self.run_static_fn = self.run_v1_fn or self._fn("forgetune_run", _RUN4, ctypes.c_int)
            if self.run_static_fn is None:
                raise ForgeTuneRuntimeError("Missing static entry point in %s" % self.original_dll_path)
            self.run_fn = self.run_static_fn
            if self.run_v1_fn is None:
                self.run_v1_fn = self.run_static_fn
        self.benchmark_fn = self._fn("forgetune_benchmark_kernel", _RUN4[:4] + [ctypes.c_int], ctypes.c_double)
        self.run_device_fn = self._fn("forgetune_run_v2_device", _RUN5 + [ctypes.c_void_p], ctypes.c_int)

    # ------------------------------------------------------------------ checks
    def _check_open(self):
        if self.is_closed:
            raise ForgeTuneRuntimeError("Cannot execute NativeRuntime after it has been closed.")

    @staticmethod
    def _as_f32(x) -> np.ndarray:
        if type(x) is not np.ndarray:
            x = np.asarray(x)
        if np.iscomplexobj(x) or x.dtype != np.float32:
            raise TypeError("Unsupported input tensor dtype '%s': ForgeTune requires float32 input "
                            "(no silent casting from '%s')." % (x.dtype, x.dtype))
        return x

    def _dynamic_batch(self, x: np.ndarray, batch_size) -> int:
        if x.ndim != len(self.expected_input_shape):
            raise InvalidShapeError("Input rank mismatch: expected %dD, got %dD"
                                    % (len(self.expected_input_shape), x.ndim))
        for d in range(1, len(self.expected_input_shape)):
            if self.expected_input_shape[d] != -1 and x.shape[d] != self.expected_input_shape[d]:
                raise InvalidShapeError("Input dimension %d mismatch: expected %d, got %d"
                                        % (d, self.expected_input_shape[d], x.shape[d]))
        b = x.shape[0]
        if batch_size is not None:
            bv = _positive_int(batch_size, "batch_size", InvalidShapeError)
            if bv != b:
                raise InvalidShapeError("Explicit batch_size %d does not match input leading dimension %d" % (bv, b))
        if b <= 0 or b > self.max_batch_size:
            raise InvalidShapeError("Dynamic batch size %d out of valid range [1, %d]" % (b, self.max_batch_size))
        return b

    def _raise_status(self, status: int, detail: str) -> None:
        msg = _STATUS.get(status, "Unknown native error code: %d" % status)
        raise ForgeTuneRuntimeError("Native kernel execution failed with code %d: %s (%s)" % (status, msg, detail))

    # ------------------------------------------------------------------ run
    def run(self, input_tensor, batch_size: Optional[int] = None) -> np.ndarray:
        """Run the model on a float32 host array; returns a new float32 array."""
        self._check_open()
        x = self._as_f32(input_tensor)
        if self.is_dynamic:
            b = self._dynamic_batch(x, batch_size)
            if not x.flags["C_CONTIGUOUS"]:
                x = np.ascontiguousarray(x)
            out_shape = (b,) + self._output_shape_tail if self.is_output_dynamic else self.expected_output_shape
            y = np.empty(out_shape, dtype=np.float32)
            if self.run_dynamic_fn is not None:
                st = self.run_dynamic_fn(x.ctypes.data, x.size, y.ctypes.data, y.size, b)
            else:
                st = self.run_v1_dynamic_fn(x.ctypes.data, x.size, y.ctypes.data, y.size)
            if st != 0:
                self._raise_status(st, "batch=%d" % b)
            return y
        if batch_size is not None:
            bv = _positive_int(batch_size, "batch_size", InvalidShapeError)
            eb = self.expected_input_shape[0] if self.expected_input_shape else 1
            if bv != eb:
                raise InvalidShapeError("Explicit batch_size %d does not match static model expected batch %d"
                                        % (bv, eb))
        if tuple(x.shape) != self.expected_input_shape:
            raise InvalidShapeError("Input shape mismatch: expected %s, got %s" % (self.expected_input_shape, x.shape))
        if not x.flags["C_CONTIGUOUS"]:
            x = np.ascontiguousarray(x)
        y = np.empty(self.expected_output_shape, dtype=np.float32)
        st = self.run_static_fn(x.ctypes.data, self.total_input_count, y.ctypes.data, self.total_output_count)
        if st != 0:
            self._raise_status(st, "static batch")
        return y

    def run_device(self, d_input: int, d_output: int, batch_size: int, stream: int = 0) -> None:
        """Run on device buffers (raw CUDA pointers) enqueued on ``stream``; does not synchronise."""
        self._check_open()
        if self.run_device_fn is None:
            raise ForgeTuneRuntimeError("library does not export forgetune_run_v2_device")
        b = _positive_int(batch_size, "batch_size", InvalidShapeError)
        fi = int(math.prod(self.expected_input_shape[1:])) if self.is_dynamic else self.total_input_count
        fo = int(math.prod(self._output_shape_tail)) if self.is_output_dynamic else self.total_output_count
        ic = b * fi if self.is_dynamic else fi
        oc = b * fo if self.is_output_dynamic else fo
        st = self.run_device_fn(d_input, ic, d_output, oc, b, stream)
        if st != 0:
            self._raise_status(st, "device run, batch=%d" % b)

    def benchmark_kernel(self, input_tensor, iters: int = 1000) -> float:
        """Average device time of one forward pass in microseconds (CUDA events)."""
        if type(iters) is not int or isinstance(iters, bool) or iters <= 0:
            raise ValueError("iters must be a positive non-boolean integer, got %r (%s)" % (iters, type(iters).__name__))
        self._check_open()
        x = self._as_f32(input_tensor)
        if self.benchmark_fn is None:
            raise ForgeTuneRuntimeError("DLL does not export forgetune_benchmark_kernel")
        if self.is_dynamic:
            b = self._dynamic_batch(x, None)
            out_shape = (b,) + self._output_shape_tail if self.is_output_dynamic else self.expected_output_shape
        else:
            if tuple(x.shape) != self.expected_input_shape:
                raise InvalidShapeError("Input shape mismatch: expected %s, got %s"
                                        % (self.expected_input_shape, x.shape))
            out_shape = self.expected_output_shape
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.empty(out_shape, dtype=np.float32)
        lat = self.benchmark_fn(x.ctypes.data, x.size, y.ctypes.data, y.size, iters)
        if not math.isfinite(lat) or lat < 0:
            raise ForgeTuneRuntimeError("Native benchmark returned invalid latency: %s (%s)" % (lat, self.last_error()))
        return float(lat)

    # ------------------------------------------------------------------ counters
    def _call(self, name: str, restype=ctypes.c_size_t, argtypes=(), args=()):
        self._check_open()
        if not hasattr(self.lib, name):
            raise ForgeTuneRuntimeError("Shared library %s does not export '%s'" % (self.original_dll_path, name))
        f = getattr(self.lib, name)
        f.restype = restype
        f.argtypes = list(argtypes)
        return f(*args)

    def get_arena_alloc_count(self) -> int:
        return int(self._call("forgetune_get_arena_alloc_count"))

    def get_arena_payload_alloc_count(self) -> int:
        return int(self._call("forgetune_get_arena_payload_alloc_count"))

    def get_arena_block_insertion_count(self) -> int:
        return int(self._call("forgetune_get_arena_block_insertion_count"))

    def get_process_arena_total_allocations(self) -> int:
        return int(self._call("forgetune_get_process_arena_total_allocations"))

    def reset_arena_alloc_count(self) -> None:
        self._call("forgetune_reset_arena_alloc_count", restype=None)

    def inject_test_arena_alloc(self) -> None:
        self._call("forgetune_test_inject_arena_alloc", restype=None)

    # ------------------------------------------------------------------ additions
    def create(self) -> None:
        st = self._call("forgetune_create", restype=ctypes.c_int)
        if st != 0:
            self._raise_status(st, "create: " + self.last_error())

    def set_devices(self, device_ids: Sequence[int]) -> None:
        arr = (ctypes.c_int * max(1, len(device_ids)))(*device_ids)
        st = self._call("forgetune_set_devices", ctypes.c_int, [ctypes.c_void_p, ctypes.c_int],
                        [ctypes.cast(arr, ctypes.c_void_p), len(device_ids)])
        if st != 0:
            self._raise_status(st, "set_devices: " + self.last_error())

    def set_kernel_policy(self, policy: int) -> None:
        st = self._call("forgetune_set_kernel_policy", ctypes.c_int, [ctypes.c_int], [int(policy)])
        if st != 0:
            self._raise_status(st, "set_kernel_policy")

    def describe(self) -> dict:
        n = self._call("forgetune_describe", ctypes.c_int, [ctypes.c_void_p, ctypes.c_size_t], [None, 0])
        if n < 0:
            self._raise_status(n, "describe")
        buf = ctypes.create_string_buffer(n + 1)
        self._call("forgetune_describe", ctypes.c_int, [ctypes.c_void_p, ctypes.c_size_t], [buf, n + 1])
        return json.loads(buf.value.decode())

    @staticmethod
    def last_error() -> str:
        from . import _native
        return _native.last_error()

    # ------------------------------------------------------------------ lifetime
    def close(self) -> None:
        """Release device resources and unload the library."""
        if self.is_closed:
            return
        self.is_closed = True
        for a in ("run_fn", "run_dynamic_fn", "run_v1_dynamic_fn", "run_static_fn", "run_v1_fn", "run_v2_fn",
                  "benchmark_fn", "run_device_fn"):
            setattr(self, a, None)
        self.unload_error = None
        lib = getattr(self, "lib", None)
        if lib is not None and getattr(lib, "_handle", None):
            try:
                if hasattr(lib, "forgetune_destroy"):
                    lib.forgetune_destroy.restype = None
                    lib.forgetune_destroy()
                import _ctypes
                _ctypes.dlclose(lib._handle)
            except Exception as ex:  # pragma: no cover - platform specific
                self.unload_error = str(ex)
        self.lib = None

    def __enter__(self):
        return self

    def __exit__(self, exc_type, exc, tb):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
