"""Exception hierarchy, with the names and bases of the reference's
(python/forgetune/errors.py:7-69) so callers' ``except`` clauses keep working."""

import builtins


class ForgeTuneError(Exception):
    """Base class for every error this package raises."""


class UnsupportedOpError(ForgeTuneError):
    def __init__(self, op_name: str, node_info: str = ""):
        self.op_name = op_name
        self.node_info = node_info
        msg = "Unsupported operator '%s'" % op_name
        if node_info:
            msg += ": " + node_info
        super().__init__(msg)


class InvalidGraphError(ForgeTuneError):
    """The exported graph cannot be lowered or fails verification."""


class InvalidShapeError(InvalidGraphError):
    """A tensor shape or batch size is outside what the compiled model accepts."""


class CodeGenError(ForgeTuneError):
    """Emitting the per-model artifact failed."""


class CompilationError(ForgeTuneError):
    def __init__(self, message: str, stdout: str = "", stderr: str = "", command: list = None):
        self.stdout = stdout
        self.stderr = stderr
        self.command = command or []
        super().__init__(message)


class CorrectnessError(ForgeTuneError):
    def __init__(self, message: str, max_abs_diff: float = 0.0, max_rel_diff: float = 0.0):
        self.max_abs_diff = max_abs_diff
        self.max_rel_diff = max_rel_diff
        super().__init__(message)


class AutotuningError(ForgeTuneError):
    """No candidate passed the correctness gate, or timing failed."""


class ForgeTuneRuntimeError(ForgeTuneError, builtins.RuntimeError):
    """A native call failed at run time."""
