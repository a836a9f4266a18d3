"""B200-native (sm_100a) execution backend for Emmy Kernel-IR KernelOps.

Drop-in for vedantgpt/emmy-ptx-compiler's ``compile.py`` surface:
``compile_ir``, ``compile_bundle`` and ``Compiler`` take the same IR JSON,
meta.json and KernelOp objects and produce one ``.visible .entry`` named after
``KernelOp.name`` with parameters in ``meta.json`` ``arg_order``, targeting
``sm_100a``.  :mod:`.runtime` launches the result through the C-ABI library
``libemmy_b200.so``.
"""

from .errors import ToolchainError, UnsupportedIR  # noqa: F401

__all__ = ["UnsupportedIR", "ToolchainError"]
