"""Errors raised by the compiler front-end and lowering.

The reference prints a one-line reason on stderr and exits 2 for any IR it
cannot lower (compile.py:1516-1518, 2196-2198, 2724-2725); the CLI maps
:class:`UnsupportedIR` to that behaviour.
"""


class UnsupportedIR(Exception):
    """The KernelOp (or an op, node or expression in it) has no lowering."""


class ToolchainError(RuntimeError):
    """nvcc/ptxas failed on generated CUDA source."""
