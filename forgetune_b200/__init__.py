"""forgetune_b200: a B200 (sm_100a) backend for ForgeTune's compiled forward pass.

``compile_model`` lowers a torch model, fuses and plans it in the native
engine, and returns a :class:`CompiledModel` whose per-model shared library
exports the reference's C ABI and runs on hand-written CUDA kernels.
``compile_graph_json`` does the same for a graph the reference's frontend or
CLI wrote to ``graph.json``; ``Autotuner`` chooses the kernels on the GPU.
"""

from .autotuner import Autotuner
from .compiler import CompiledModel, compile_graph_json, compile_model
from .errors import (AutotuningError, CodeGenError, CompilationError, CorrectnessError, ForgeTuneError,
                     ForgeTuneRuntimeError, InvalidGraphError, InvalidShapeError, UnsupportedOpError)
from .frontend import IRGraph, export_to_ir
from .ir_json import load_graph_json, to_graph_json
from .runtime import NativeRuntime

__version__ = "0.1.0"
__all__ = [
    "compile_model", "compile_graph_json", "CompiledModel", "NativeRuntime", "IRGraph", "export_to_ir",
    "load_graph_json", "to_graph_json", "Autotuner",
    "ForgeTuneError", "UnsupportedOpError", "InvalidGraphError", "InvalidShapeError", "CodeGenError",
    "CompilationError", "CorrectnessError", "AutotuningError", "ForgeTuneRuntimeError",
]
