"""ctypes binding of ``libemmy_b200.so`` (C ABI: include/emmy_b200.h).

This is the launch side the reference leaves to its external runner
(README.md:170-182): load the module for a KernelOp, launch its entry on
device buffers in ``arg_order``, read back the kernel status word.  There is
no CPU fallback: if the library or a GPU is missing, calls raise
:class:`EmmyError`.
"""

from __future__ import annotations

import ctypes as C
import struct
import threading
from pathlib import Path

from . import native

EMMY_ROLE_IN, EMMY_ROLE_OUT, EMMY_ROLE_INOUT, EMMY_ROLE_OUT_ZEROED, EMMY_ROLE_SCALAR = 0, 1, 2, 3, 4
FAMILY_NAMES = {0: "foreign", 1: "pointwise", 2: "reduction", 3: "gemm", 4: "rownorm", 5: "attention",
                6: "schedule"}

_lock = threading.Lock()
_lib = None
_initialised: set[int] = set()


class EmmyError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"emmy error {code}: {msg}")
        self.code = code


def _declare(lib) -> None:
    u64, u32, i32, vp, sz = C.c_uint64, C.c_uint32, C.c_int, C.c_void_p, C.c_size_t
    P = C.POINTER
    sigs = {
        "emmy_version": ([], C.c_char_p),
        "emmy_last_error": ([C.c_char_p, sz], i32),
        "emmy_init": ([i32], i32),
        "emmy_device_count": ([P(i32)], i32),
        "emmy_load": ([i32, vp, sz, C.c_char_p, P(vp)], i32),
        "emmy_unload": ([vp], i32),
        "emmy_module_info": ([vp, P(u32), P(u32), P(u32), P(u32), P(u32)], i32),
        "emmy_launch": ([vp, P(u64), i32, P(u32), P(u32), u64], i32),
        "emmy_launch_ex": ([vp, P(u64), i32, P(u32), P(u32), u32, u64], i32),
        "emmy_module_status": ([vp, P(u32)], i32),
        "emmy_sync": ([i32, u64, i32], i32),
        "emmy_alloc": ([i32, sz, P(u64)], i32),
        "emmy_free": ([i32, u64], i32),
        "emmy_memcpy_htod": ([i32, u64, vp, sz, u64], i32),
        "emmy_memcpy_dtoh": ([i32, vp, u64, sz, u64], i32),
        "emmy_memset_d8": ([i32, u64, C.c_uint8, sz, u64], i32),
        "emmy_host_alloc": ([sz, P(vp)], i32),
        "emmy_host_free": ([vp], i32),
        "emmy_run_host": ([vp, P(vp), P(sz), P(C.c_uint8), i32, u64], i32),
        "emmy_time_launch": ([vp, P(u64), i32, i32, u64, P(C.c_float)], i32),
        "emmy_launch_range": ([vp, P(u64), i32, u64, u64, u64], i32),
        "emmy_module_range": ([vp, P(u64), P(u32), P(u64), i32], i32),
        "emmy_shard_range": ([vp, i32, i32, P(u64), P(u64)], i32),
        "emmy_launch_sharded": ([P(vp), i32, P(P(u64)), i32, P(u64)], i32),
        "emmy_sum_f32_noalloc": ([i32, u64, u64, u64, u64], i32),
        "emmy_xchg_create": ([i32, i32, i32, P(vp), P(C.c_uint8)], i32),
        "emmy_xchg_connect": ([vp, P(C.c_uint8)], i32),
        "emmy_sum_f32_allreduce": ([vp, u64, u64, u64, i32, u64], i32),
        "emmy_xchg_status": ([vp, P(u32)], i32),
        "emmy_xchg_reset": ([vp], i32),
        "emmy_launch_xchg": ([vp, P(u64), i32, vp, i32, u64], i32),
        "emmy_xchg_destroy": ([vp], i32),
        "emmy_comm_unique_id": ([P(C.c_uint8)], i32),
        "emmy_comm_init": ([i32, i32, i32, P(C.c_uint8), i32, P(vp)], i32),
        "emmy_allreduce_f32": ([vp, u64, u64, sz, u64, i32], i32),
        "emmy_allgather_f32": ([vp, u64, u64, sz, u64, i32], i32),
        "emmy_comm_destroy": ([vp], i32),
        "emmy_comm_abort": ([vp], i32),
        "emmy_graph_begin": ([i32, u64], i32),
        "emmy_graph_end": ([i32, u64, P(vp)], i32),
        "emmy_graph_launch": ([vp, u64], i32),
        "emmy_graph_destroy": ([vp], i32),
    }
    for name, (argtypes, restype) in sigs.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = restype


EXPORTED = ("emmy_version", "emmy_last_error", "emmy_init", "emmy_device_count", "emmy_load",
            "emmy_unload", "emmy_module_info", "emmy_launch", "emmy_launch_ex", "emmy_module_status", "emmy_sync",
            "emmy_alloc", "emmy_free", "emmy_memcpy_htod", "emmy_memcpy_dtoh", "emmy_memset_d8",
            "emmy_host_alloc", "emmy_host_free", "emmy_run_host", "emmy_time_launch", "emmy_launch_range",
            "emmy_module_range", "emmy_shard_range", "emmy_launch_sharded", "emmy_sum_f32_noalloc",
            "emmy_xchg_create", "emmy_xchg_connect", "emmy_sum_f32_allreduce", "emmy_xchg_status",
            "emmy_xchg_reset", "emmy_launch_xchg", "emmy_xchg_destroy",
            "emmy_comm_unique_id", "emmy_comm_init", "emmy_allreduce_f32", "emmy_allgather_f32",
            "emmy_comm_destroy", "emmy_comm_abort",
            "emmy_graph_begin", "emmy_graph_end", "emmy_graph_launch", "emmy_graph_destroy")


def library_path() -> Path:
    return native.RUNTIME_SO


def lib():
    """Load (building first if needed) the native library."""
    global _lib
    with _lock:
        if _lib is None:
            path = native.build_runtime()
            handle = C.CDLL(str(path), mode=C.RTLD_GLOBAL)
            _declare(handle)
            _lib = handle
        return _lib


def _check(rc: int) -> None:
    if rc != 0:
        buf = C.create_string_buffer(2048)
        lib().emmy_last_error(buf, len(buf))
        raise EmmyError(rc, buf.value.decode(errors="replace"))


def init(device: int = 0) -> None:
    """Initialise devices [0, device] (their primary contexts)."""
    if device in _initialised:
        return
    _check(lib().emmy_init(device + 1))
    _initialised.update(range(device + 1))


def device_count() -> int:
    n = C.c_int(0)
    _check(lib().emmy_device_count(C.byref(n)))
    return n.value


def arg_word(value) -> int:
    """One 64-bit launch word: device pointer, torch tensor, f32 or i32 scalar."""
    if hasattr(value, "data_ptr"):
        return int(value.data_ptr())
    if isinstance(value, float):
        return struct.unpack("<I", struct.pack("<f", value))[0]
    if isinstance(value, int):
        return value & 0xFFFFFFFFFFFFFFFF
    if isinstance(value, tuple) and len(value) == 2 and value[0] == "i32":
        return int(value[1]) & 0xFFFFFFFF
    raise TypeError(f"cannot pass {type(value).__name__} as a kernel argument")


class Module:
    """One loaded entry on one device."""

    def __init__(self, image: bytes, entry: str, device: int = 0):
        init(device)
        self.device = device
        self.entry = entry
        self._image = image
        h = C.c_void_p()
        _check(lib().emmy_load(device, image, len(image), entry.encode(), C.byref(h)))
        self._h = h
        fam, nparams, smem = C.c_uint32(), C.c_uint32(), C.c_uint32()
        grid, block = (C.c_uint32 * 3)(), (C.c_uint32 * 3)()
        _check(lib().emmy_module_info(h, C.byref(fam), grid, block, C.byref(smem), C.byref(nparams)))
        self.family = FAMILY_NAMES.get(fam.value, str(fam.value))
        self.grid = tuple(grid)
        self.block = tuple(block)
        self.smem = smem.value
        self.nparams = nparams.value

    def close(self) -> None:
        if getattr(self, "_h", None):
            _check(lib().emmy_unload(self._h))
            self._h = None

    def __del__(self):  # best effort; explicit close() is preferred
        try:
            if getattr(self, "_h", None) and _lib is not None:
                _lib.emmy_unload(self._h)
        except Exception:
            pass

    def _words(self, args) -> C.Array:
        return (C.c_uint64 * max(1, len(args)))(*[arg_word(a) for a in args])

    def launch(self, args, stream: int = 0, grid=None, block=None, smem: int | None = None) -> None:
        """``smem``: dynamic shared-memory bytes for an explicit ``grid``/``block``
        launch (the meta.json ``smem_bytes``); None keeps the module's own."""
        words = self._words(args)
        g = (C.c_uint32 * 3)(*(list(grid) + [1, 1])[:3]) if grid is not None else None
        b = (C.c_uint32 * 3)(*(list(block) + [1, 1])[:3]) if block is not None else None
        if smem is not None:
            _check(lib().emmy_launch_ex(self._h, words, len(args), g, b, C.c_uint32(int(smem)), C.c_uint64(stream)))
            return
        _check(lib().emmy_launch(self._h, words, len(args), g, b, C.c_uint64(stream)))

    def bind(self, args, stream: int = 0) -> "BoundLaunch":
        """A launcher with the argument words prepared once (the tensors must
        stay alive and keep their storage): each call is one C-ABI launch."""
        return BoundLaunch(self, self._words(args), len(args), stream)

    def launch_range(self, args, begin: int, end: int, stream: int = 0) -> None:
        """Launch over units [begin, end) (cells / output rows) only."""
        words = self._words(args)
        _check(lib().emmy_launch_range(self._h, words, len(args), C.c_uint64(begin), C.c_uint64(end),
                                       C.c_uint64(stream)))

    def unit_range(self) -> tuple[int, int, list[int]]:
        """(total units, alignment, bytes per unit of each parameter); total 0 = no ranges."""
        tot, al = C.c_uint64(0), C.c_uint32(0)
        per = (C.c_uint64 * 32)()
        _check(lib().emmy_module_range(self._h, C.byref(tot), C.byref(al), per, 32))
        return tot.value, al.value, list(per)[: self.nparams]

    def status(self) -> int:
        st = C.c_uint32(0)
        _check(lib().emmy_module_status(self._h, C.byref(st)))
        return st.value

    def time(self, args, iters: int, stream: int = 0) -> float:
        """Total device milliseconds of ``iters`` back-to-back launches."""
        words = self._words(args)
        ms = C.c_float(0.0)
        _check(lib().emmy_time_launch(self._h, words, len(args), iters, C.c_uint64(stream), C.byref(ms)))
        return ms.value

    def run_host(self, host_ptrs: list[int], nbytes: list[int], roles: list[int], stream: int = 0) -> None:
        n = len(host_ptrs)
        ptrs = (C.c_void_p * n)(*host_ptrs)
        sizes = (C.c_size_t * n)(*nbytes)
        rl = (C.c_uint8 * n)(*roles)
        _check(lib().emmy_run_host(self._h, ptrs, sizes, rl, n, C.c_uint64(stream)))


class BoundLaunch:
    """``Module.launch`` with fixed arguments and stream, for launch-rate-bound
    loops: the call does no Python-side argument marshalling."""

    def __init__(self, module: Module, words, nargs: int, stream: int):
        self._module = module  # keeps the module loaded
        self._fn = lib().emmy_launch
        self._h = module._h
        self._words = words
        self._nargs = nargs
        self._stream = C.c_uint64(stream)

    def __call__(self) -> None:
        rc = self._fn(self._h, self._words, self._nargs, None, None, self._stream)
        if rc:
            _check(rc)


class Graph:
    """A CUDA graph of the launches issued on one stream between
    ``begin`` and ``end`` (``with Graph.record(dev, stream) as g: ...``);
    ``launch`` replays them in order, with the recorded arguments."""

    def __init__(self, device: int):
        self.device = device
        self._h = None

    @classmethod
    def record(cls, device: int, stream: int) -> "_Recording":
        return _Recording(cls(device), stream)

    def launch(self, stream: int) -> None:
        if not self._h:
            raise EmmyError(-1, "graph has not been recorded")
        _check(lib().emmy_graph_launch(self._h, C.c_uint64(stream)))

    def close(self) -> None:
        if self._h:
            h, self._h = self._h, None
            _check(lib().emmy_graph_destroy(h))

    def __del__(self):
        try:
            if self._h and _lib is not None:
                _lib.emmy_graph_destroy(self._h)
        except Exception:
            pass


class _Recording:
    def __init__(self, graph: Graph, stream: int):
        self.graph, self.stream = graph, stream

    def __enter__(self) -> Graph:
        _check(lib().emmy_graph_begin(self.graph.device, C.c_uint64(self.stream)))
        return self.graph

    def __exit__(self, exc_type, exc, tb) -> None:
        h = C.c_void_p()
        rc = lib().emmy_graph_end(self.graph.device, C.c_uint64(self.stream), C.byref(h))
        if exc_type is None:
            _check(rc)
            self.graph._h = h
        elif h:
            lib().emmy_graph_destroy(h)


def shard_range(module: "Module", ndev: int, d: int) -> tuple[int, int]:
    """Units [begin, end) that device ``d`` of ``ndev`` processes in a sharded launch."""
    b, e = C.c_uint64(0), C.c_uint64(0)
    _check(lib().emmy_shard_range(module._h, ndev, d, C.byref(b), C.byref(e)))
    return b.value, e.value


def launch_sharded(modules: list["Module"], args_per_device: list[list], streams: list[int] | None = None) -> None:
    """One launch split by unit range over the devices of ``modules`` (one
    module per device); streamed parameters are each device's shard."""
    n = len(modules)
    mods = (C.c_void_p * n)(*[m._h.value for m in modules])
    words = [(C.c_uint64 * max(1, len(a)))(*[arg_word(x) for x in a]) for a in args_per_device]
    arr = (C.POINTER(C.c_uint64) * n)(*[C.cast(w, C.POINTER(C.c_uint64)) for w in words])
    st = (C.c_uint64 * n)(*(streams or [0] * n))
    _check(lib().emmy_launch_sharded(mods, n, arr, len(args_per_device[0]), st))


class Exchange:
    """This GPU's end of the fused sum + cross-GPU combine (emmy_xchg_*):
    ``Exchange(dev, nranks, rank)``, pass every rank's ``handle`` (in rank
    order) to ``connect``, then ``sum_allreduce``."""

    HANDLE_BYTES = 64

    def __init__(self, device: int, nranks: int, rank: int):
        init(device)
        self.device = device
        h = C.c_void_p()
        buf = (C.c_uint8 * self.HANDLE_BYTES)()
        _check(lib().emmy_xchg_create(device, nranks, rank, C.byref(h), buf))
        self._h = h
        self.handle = bytes(buf)

    def connect(self, handles: list[bytes]) -> None:
        blob = b"".join(handles)
        arr = (C.c_uint8 * len(blob)).from_buffer_copy(blob)
        _check(lib().emmy_xchg_connect(self._h, arr))

    def sum_allreduce(self, x, n: int, out, timeout_ms: int = 1000, stream: int = 0) -> None:
        _check(lib().emmy_sum_f32_allreduce(self._h, C.c_uint64(arg_word(x)), C.c_uint64(n),
                                            C.c_uint64(arg_word(out)), timeout_ms, C.c_uint64(stream)))

    def launch(self, module: "Module", args, timeout_ms: int = 1000, stream: int = 0) -> None:
        """One launch of ``module``'s cross-GPU entry (a compiled full-array
        reduction): this GPU's shard reduced, every GPU's result combined."""
        words = module._words(args)
        _check(lib().emmy_launch_xchg(module._h, words, len(args), self._h, timeout_ms, C.c_uint64(stream)))

    def bind(self, module: "Module", args, timeout_ms: int = 1000, stream: int = 0):
        """A no-argument callable for ``launch`` with the words prepared once."""
        words = module._words(args)
        n, h, mh, f = len(args), self._h, module._h, lib().emmy_launch_xchg
        st = C.c_uint64(stream)

        def go() -> None:
            rc = f(mh, words, n, h, timeout_ms, st)
            if rc:
                _check(rc)
        return go

    def status(self) -> int:
        st = C.c_uint32(0)
        _check(lib().emmy_xchg_status(self._h, C.byref(st)))
        return st.value

    def reset(self) -> None:
        """Clear the group after a failed call (every rank, nothing in flight)."""
        _check(lib().emmy_xchg_reset(self._h))

    def close(self) -> None:
        if getattr(self, "_h", None):
            _check(lib().emmy_xchg_destroy(self._h))
            self._h = None


def sum_f32_noalloc(x, n: int, out, device: int = 0, stream: int = 0) -> None:
    """``out[0] = sum(x[:n])`` through emmy_sum_f32_noalloc: no device memory is
    allocated; cross-block partials live in the library's fixed scratch array
    (calls overlapping on one GPU race on it)."""
    init(device)
    _check(lib().emmy_sum_f32_noalloc(device, arg_word(x), n, arg_word(out), stream))


def sync(device: int = 0, stream: int = 0, timeout_ms: int = 0) -> None:
    _check(lib().emmy_sync(device, C.c_uint64(stream), timeout_ms))


class Comm:
    """NCCL communicator for the per-GPU partial combine of full reductions."""

    @staticmethod
    def unique_id() -> bytes:
        buf = (C.c_uint8 * 128)()
        _check(lib().emmy_comm_unique_id(buf))
        return bytes(buf)

    def __init__(self, device: int, nranks: int, rank: int, uid: bytes, timeout_ms: int = 60000):
        init(device)
        self.device = device
        h = C.c_void_p()
        idbuf = (C.c_uint8 * 128)(*uid)
        _check(lib().emmy_comm_init(device, nranks, rank, idbuf, timeout_ms, C.byref(h)))
        self._h = h

    def allreduce_f32(self, send: int, recv: int, count: int, stream: int = 0, timeout_ms: int = 60000) -> None:
        _check(lib().emmy_allreduce_f32(self._h, send, recv, count, C.c_uint64(stream), timeout_ms))

    def allgather_f32(self, send: int, recv: int, count: int, stream: int = 0, timeout_ms: int = 60000) -> None:
        _check(lib().emmy_allgather_f32(self._h, send, recv, count, C.c_uint64(stream), timeout_ms))

    def close(self) -> None:
        if self._h:
            _check(lib().emmy_comm_destroy(self._h))
            self._h = None

    def abort(self) -> None:
        if self._h:
            lib().emmy_comm_abort(self._h)
            self._h = None
