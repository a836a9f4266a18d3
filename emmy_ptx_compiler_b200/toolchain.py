"""nvcc driver with an on-disk cache of built modules.

Generated family sources are compiled for ``sm_100a`` only (tcgen05 and the
GEMM family's TMA paths need the arch-specific target).  Results are cached
by a hash of source + flags + nvcc version, in ``EMMY_KCACHE`` or the
package's ``_kcache`` directory, so tests and benchmarks pay nvcc once per
distinct kernel.
"""

from __future__ import annotations

import hashlib
import json
import os
import re
import shutil
import subprocess
import tempfile
import threading
from functools import lru_cache
from pathlib import Path

from .errors import ToolchainError

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
INCLUDE_DIRS = [REPO / "include", PKG / "csrc"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--fmad=false", "-Xptxas", "-O3"]


def nvcc_path() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise ToolchainError("nvcc not found (CUDA 12.9 toolkit expected)")
    return found


@lru_cache(maxsize=1)
def nvcc_version() -> str:
    out = subprocess.run([nvcc_path(), "--version"], capture_output=True, text=True, check=False)
    return out.stdout.strip().splitlines()[-1] if out.stdout else "unknown"


def cache_dir() -> Path:
    d = Path(os.environ.get("EMMY_KCACHE", PKG / "_kcache"))
    d.mkdir(parents=True, exist_ok=True)
    return d


def _key(source: str, kind: str, extra: list[str]) -> str:
    h = hashlib.sha256()
    for part in (source, kind, " ".join(ARCH_FLAGS + COMMON_FLAGS + extra), nvcc_version()):
        h.update(part.encode())
        h.update(b"\0")
    for inc in INCLUDE_DIRS:
        for f in sorted(inc.glob("*.h*")):
            h.update(f.read_bytes())
    return h.hexdigest()[:24]


def build(source: str, kind: str = "ptx", extra: list[str] | None = None, name: str = "kernel") -> bytes:
    """Compile ``source`` to ``kind`` ("ptx" or "cubin") and return the bytes."""
    if kind not in ("ptx", "cubin"):
        raise ValueError(kind)
    extra = list(extra or [])
    key = _key(source, kind, extra)
    out_path = cache_dir() / f"{name}-{key}.{kind}"
    if out_path.is_file():
        return out_path.read_bytes()
    with tempfile.TemporaryDirectory(prefix="emmy_nvcc_") as td:
        src = Path(td) / f"{name}.cu"
        src.write_text(source)
        dst = Path(td) / f"{name}.{kind}"
        cmd = [nvcc_path(), *ARCH_FLAGS, *COMMON_FLAGS, *extra, f"-{kind}",
               *[f"-I{d}" for d in INCLUDE_DIRS], "-o", str(dst), str(src)]
        proc = subprocess.run(cmd, capture_output=True, text=True, check=False)
        if proc.returncode != 0:
            raise ToolchainError(f"nvcc failed ({proc.returncode}) on {name}:\n{proc.stderr[-4000:]}")
        data = dst.read_bytes()
    # unique per process and thread: two threads may build the same source at once
    tmp = out_path.with_suffix(out_path.suffix + f".tmp{os.getpid()}.{threading.get_ident()}")
    tmp.write_bytes(data)
    os.replace(tmp, out_path)
    return data


def resource_usage(source: str, name: str = "kernel") -> str:
    """``ptxas -v`` report (registers, spills, shared memory) for ``source``."""
    with tempfile.TemporaryDirectory(prefix="emmy_nvcc_") as td:
        src = Path(td) / f"{name}.cu"
        src.write_text(source)
        cmd = [nvcc_path(), *ARCH_FLAGS, *COMMON_FLAGS, "-Xptxas", "-v", "-cubin",
               *[f"-I{d}" for d in INCLUDE_DIRS], "-o", str(Path(td) / "k.cubin"), str(src)]
        proc = subprocess.run(cmd, capture_output=True, text=True, check=False)
        if proc.returncode != 0:
            raise ToolchainError(proc.stderr[-4000:])
        return proc.stderr


def register_usage(source: str, name: str = "kernel") -> dict:
    """Registers, barriers and spill bytes per entry of ``source`` as
    ``ptxas -v`` reports them for sm_100a, cached like the builds."""
    key = _key(source, "ptxas-v", [])
    path = cache_dir() / f"{name}-{key}.regs.json"
    if path.is_file():
        return json.loads(path.read_text())
    out: dict[str, dict] = {}
    cur = None
    for line in resource_usage(source, name).splitlines():
        m = re.search(r"Compiling entry function '([^']+)'", line)
        if m:
            cur = out.setdefault(m.group(1), {})
            continue
        if cur is None:
            continue
        m = re.search(r"Used (\d+) registers", line)
        if m:
            cur["registers"] = int(m.group(1))
            b = re.search(r"used (\d+) barriers", line)
            if b:
                cur["barriers"] = int(b.group(1))
        m = re.search(r"(\d+) bytes spill stores, (\d+) bytes spill loads", line)
        if m:
            cur["spill_stores"], cur["spill_loads"] = int(m.group(1)), int(m.group(2))
    tmp = path.with_suffix(path.suffix + f".tmp{os.getpid()}.{threading.get_ident()}")
    tmp.write_text(json.dumps(out))
    os.replace(tmp, path)
    return out
