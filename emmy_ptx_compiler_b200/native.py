"""Build recipe for the in-tree native library ``lib/libemmy_b200.so``.

The launcher is plain C++ over the CUDA driver API (libcuda and libnccl are
opened at run time); the one precompiled kernel of the library
(csrc/emmy_noalloc.cu) is built with nvcc for sm_100a and uses a private,
statically linked CUDA runtime.  The library builds and loads on machines
without a GPU.
"""

from __future__ import annotations

import os
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
LIB_DIR = PKG / "lib"
RUNTIME_SO = LIB_DIR / "libemmy_b200.so"
SOURCES = [PKG / "csrc" / "emmy_runtime.cpp"]
CUDA_SOURCES = [PKG / "csrc" / "emmy_noalloc.cu", PKG / "csrc" / "emmy_xchg.cu"]
HEADERS = [REPO / "include" / "emmy_b200.h", REPO / "include" / "emmy_launch_record.h",
           PKG / "csrc" / "emmy_xchg_dev.cuh"]
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
CUDA_INC = CUDA_HOME / "include"
CUDA_LIB = CUDA_HOME / "lib64"
NVCC = str(CUDA_HOME / "bin" / "nvcc")


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.is_file():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps if d.exists())


def build_runtime(force: bool = False) -> Path:
    if not force and not _stale(RUNTIME_SO, SOURCES + CUDA_SOURCES + HEADERS):
        return RUNTIME_SO
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    tmp = RUNTIME_SO.with_suffix(f".so.tmp{os.getpid()}")
    objs = []
    for cu in CUDA_SOURCES:
        obj = LIB_DIR / (cu.stem + ".o")
        cmd = [NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-lineinfo",
               "-Xcompiler", "-fPIC", f"-I{REPO / 'include'}", "-c", str(cu), "-o", str(obj)]
        proc = subprocess.run(cmd, capture_output=True, text=True, check=False)
        if proc.returncode != 0:
            raise RuntimeError(f"compiling {cu.name} failed:\n{proc.stderr[-4000:]}")
        objs.append(str(obj))
    # the CUDA runtime is linked statically with its symbols kept private, so the
    # library loads without a driver and never interposes on another cudart
    cmd = ["g++", "-O2", "-g", "-std=c++17", "-fPIC", "-shared", "-Wall", "-Wextra",
           f"-I{REPO / 'include'}", f"-I{CUDA_INC}", "-I/usr/include",
           *[str(s) for s in SOURCES], *objs, "-o", str(tmp),
           f"-L{CUDA_LIB}", "-lcudart_static", "-Wl,--exclude-libs,ALL", "-lrt", "-ldl", "-lpthread"]
    proc = subprocess.run(cmd, capture_output=True, text=True, check=False)
    if proc.returncode != 0:
        raise RuntimeError(f"building libemmy_b200.so failed:\n{proc.stderr[-4000:]}")
    os.replace(tmp, RUNTIME_SO)
    return RUNTIME_SO


if __name__ == "__main__":
    print(build_runtime(force=True))
