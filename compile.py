#!/usr/bin/env python3
"""Kernel IR -> sm_100a PTX.  Drop-in for the reference CLI:

    python compile.py path/to/kernel.ir.json > out.ptx

stdout carries the PTX module only; diagnostics go to stderr; exit 2 on
wrong usage or an IR no kernel family lowers.
"""

import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent))

from emmy_ptx_compiler_b200.compiler import compile_bundle, compile_ir, main  # noqa: E402,F401

if __name__ == "__main__":
    raise SystemExit(main())
