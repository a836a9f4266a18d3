"""Kernel-IR data model (the Emmy ``KernelOp`` vocabulary).

The product reads Emmy Kernel IR without the ``emmy`` package: IR JSON
stores each KernelOp body as ``repr(body)`` text (the reference's fixture
tools write it that way, tools/make_proxy_set.py:49-55), and
:mod:`emmy_ptx_compiler_b200.frontend` decodes that text into the classes
below.  The classes keep Emmy's constructor signatures (positional order and
keyword names as the reference's tests and tools call them, e.g.
``Load(names, input, index, dtype)``, ``Tile(axes, body, block_threads=...)``)
so IR can also be built in Python and handed to
:class:`emmy_ptx_compiler_b200.compiler.Compiler`, exactly as the reference's
tests drive its ``Compiler`` (tests/test_peepholes.py:25-30).
"""

from __future__ import annotations

import math
from typing import Any


def _fmt(v: Any) -> str:
    if isinstance(v, float):
        if math.isnan(v):
            return "float('nan')"
        if math.isinf(v):
            return "float('inf')" if v > 0 else "float('-inf')"
        return repr(v)
    if isinstance(v, tuple):
        inner = ", ".join(_fmt(x) for x in v)
        return f"({inner},)" if len(v) == 1 else f"({inner})"
    return repr(v)


def _tup(x) -> tuple:
    if x is None:
        return ()
    if isinstance(x, (list, tuple)):
        return tuple(x)
    return (x,)


class Node:
    """Base: ``FIELDS`` gives positional order; ``DEFAULTS`` the optional ones;
    ``TUPLES`` the fields normalised to tuples; ``BODIES`` the child bodies."""

    FIELDS: tuple[str, ...] = ()
    DEFAULTS: dict[str, Any] = {}
    TUPLES: tuple[str, ...] = ()
    BODIES: tuple[str, ...] = ()

    def __init__(self, *args, **kwargs):
        cls = type(self).__name__
        if len(args) > len(self.FIELDS):
            raise TypeError(f"{cls}: expected at most {len(self.FIELDS)} positional arguments")
        vals = dict(zip(self.FIELDS, args))
        for k, v in kwargs.items():
            if k not in self.FIELDS:
                raise TypeError(f"{cls}: unknown field {k!r}")
            if k in vals:
                raise TypeError(f"{cls}: field {k!r} given twice")
            vals[k] = v
        for f in self.FIELDS:
            if f in vals:
                v = vals[f]
            elif f in self.DEFAULTS:
                v = self.DEFAULTS[f]
            else:
                raise TypeError(f"{cls}: missing field {f!r}")
            if f in self.TUPLES:
                v = _tup(v)
            setattr(self, f, v)
        self._post_init()

    def _post_init(self) -> None:
        pass

    def __repr__(self) -> str:
        return f"{type(self).__name__}(" + ", ".join(
            f"{f}={_fmt(getattr(self, f))}" for f in self.FIELDS) + ")"

    def __eq__(self, other) -> bool:
        return type(self) is type(other) and all(getattr(self, f) == getattr(other, f)
                                                 for f in self.FIELDS)

    def __hash__(self) -> int:
        return hash(repr(self))

    def nested(self) -> tuple:
        return tuple(getattr(self, b) for b in self.BODIES)


# ------------------------------------------------------------------ scalars / types


class Dim(Node):
    FIELDS = ("value",)

    def _post_init(self) -> None:
        self.value = int(self.value)

    def as_static(self) -> int:
        return self.value

    def __int__(self) -> int:
        return self.value

    def __repr__(self) -> str:
        return f"Dim({self.value})"


class DataType(Node):
    FIELDS = ("name", "np_dtype", "itemsize")
    DEFAULTS = {"np_dtype": None, "itemsize": 4}

    def __str__(self) -> str:
        return str(self.name)

    def __repr__(self) -> str:
        npd = "None" if self.np_dtype is None else f"dtype({str(self.np_dtype)!r})"
        return f"DataType(name={self.name!r}, np_dtype={npd}, itemsize={self.itemsize!r})"


class ElementwiseImpl(Node):
    FIELDS = ("name", "identity")
    DEFAULTS = {"identity": None}


class Tensor(Node):
    FIELDS = ("name", "shape", "dtype")
    DEFAULTS = {"shape": (), "dtype": "f32"}
    TUPLES = ("shape",)


# ------------------------------------------------------------------ expressions


class Expr(Node):
    def pretty(self) -> str:  # deterministic structural text
        raise NotImplementedError

    def simplify(self, ctx=None) -> "Expr":
        return self

    def var_names(self) -> set[str]:
        out: set[str] = set()
        for f in self.FIELDS:
            v = getattr(self, f)
            for item in (v if isinstance(v, tuple) else (v,)):
                if isinstance(item, Expr):
                    out |= item.var_names()
        return out


class SimplifyCtx:
    @staticmethod
    def empty() -> "SimplifyCtx":
        return SimplifyCtx()


class Var(Expr):
    FIELDS = ("name",)

    def pretty(self) -> str:
        return self.name

    def var_names(self) -> set[str]:
        return {self.name}


class Builtin(Expr):
    FIELDS = ("name",)

    def pretty(self) -> str:
        return self.name

    def var_names(self) -> set[str]:
        return {self.name}


class Literal(Expr):
    FIELDS = ("value", "dtype")
    DEFAULTS = {"dtype": None}

    def pretty(self) -> str:
        return repr(self.value)


class BinaryExpr(Expr):
    FIELDS = ("op", "left", "right")

    def pretty(self) -> str:
        return f"({self.left.pretty()} {self.op} {self.right.pretty()})"


class TernaryExpr(Expr):
    FIELDS = ("cond", "if_true", "if_false")

    def pretty(self) -> str:
        return f"({self.cond.pretty()} ? {self.if_true.pretty()} : {self.if_false.pretty()})"


class CastExpr(Expr):
    FIELDS = ("expr", "dtype")

    @property
    def value(self):
        return self.expr

    def pretty(self) -> str:
        return f"(({self.dtype}){self.expr.pretty()})"


class FuncCallExpr(Expr):
    FIELDS = ("name", "args")
    DEFAULTS = {"args": ()}
    TUPLES = ("args",)

    def pretty(self) -> str:
        return f"{self.name}(" + ", ".join(a.pretty() for a in self.args) + ")"


class FlatIndex(Expr):
    FIELDS = ("buffer", "index")
    DEFAULTS = {"index": ()}
    TUPLES = ("index",)

    def pretty(self) -> str:
        return f"flat({self.buffer}[" + ", ".join(i.pretty() for i in self.index) + "])"


# ------------------------------------------------------------------ statements


class Stmt(Node):
    def reads(self) -> set[str]:
        """IR names this statement reads (values and index variables)."""
        out: set[str] = set()
        for f in self.FIELDS:
            if f in self.BODIES:
                continue
            v = getattr(self, f)
            for item in (v if isinstance(v, tuple) else (v,)):
                if isinstance(item, Expr):
                    out |= item.var_names()
        return out


class Axis(Node):
    FIELDS = ("name", "extent")

    def _post_init(self) -> None:
        if not isinstance(self.extent, Dim):
            self.extent = Dim(int(self.extent))

    @property
    def size(self) -> int:
        return int(self.extent.value)


class KernelOp(Node):
    FIELDS = ("name", "body", "inputs", "outputs")
    DEFAULTS = {"body": (), "inputs": None, "outputs": None}
    TUPLES = ("body",)

    def _post_init(self) -> None:
        self.inputs = dict(self.inputs or {})
        self.outputs = dict(self.outputs or {})


class Tile(Stmt):
    FIELDS = ("axes", "body", "block_threads", "aux_threads", "raster_group", "raster_axes",
              "raster_orient")
    DEFAULTS = {"body": (), "block_threads": None, "aux_threads": 0, "raster_group": None,
                "raster_axes": None, "raster_orient": None}
    TUPLES = ("axes", "body")
    BODIES = ("body",)


class Smem(Stmt):
    FIELDS = ("name", "extents", "dtype", "align")
    DEFAULTS = {"dtype": "f32", "align": 0}
    TUPLES = ("extents",)


class Sync(Stmt):
    FIELDS = ("barrier_id", "count", "warp")
    DEFAULTS = {"barrier_id": 0, "count": 0, "warp": False}


class WarpShuffle(Stmt):
    FIELDS = ("state", "state_b", "combine_states", "length", "dtype")
    DEFAULTS = {"length": 32, "dtype": None}
    TUPLES = ("state", "state_b", "combine_states")

    def reads(self) -> set[str]:
        return set(self.state)


class TreeHalve(Stmt):
    FIELDS = ("bufs", "state", "state_b", "combine_states", "length", "tid_var", "inner",
              "barrier_id", "barrier_count", "dtype")
    DEFAULTS = {"inner": None, "barrier_id": 0, "barrier_count": 0, "dtype": None}
    TUPLES = ("bufs", "state", "state_b", "combine_states")

    def reads(self) -> set[str]:
        return set(self.state) | {self.tid_var}


class Load(Stmt):
    FIELDS = ("names", "input", "index", "dtype")
    DEFAULTS = {"index": (), "dtype": None}
    TUPLES = ("names", "index")


class Write(Stmt):
    FIELDS = ("output", "index", "values", "value_dtype", "atomic")
    DEFAULTS = {"index": (), "values": (), "value_dtype": None, "atomic": False}
    TUPLES = ("index", "values")

    def reads(self) -> set[str]:
        return super().reads() | set(self.values)


class Assign(Stmt):
    FIELDS = ("name", "op", "args", "dtype")
    DEFAULTS = {"args": (), "dtype": None}
    TUPLES = ("args",)

    def reads(self) -> set[str]:
        return {a for a in self.args if isinstance(a, str)}


class Accum(Stmt):
    FIELDS = ("name", "value", "op", "dtype", "axes", "base")
    DEFAULTS = {"op": None, "dtype": None, "axes": (), "base": None}
    TUPLES = ("axes",)

    def _post_init(self) -> None:
        if self.op is None:
            self.op = ElementwiseImpl("add")

    def reads(self) -> set[str]:
        return {x for x in (self.value, self.base) if isinstance(x, str)}


class Init(Stmt):
    FIELDS = ("name", "identity", "dtype")
    DEFAULTS = {"identity": 0.0, "dtype": None}


class Let(Stmt):
    FIELDS = ("name", "value", "dtype")
    DEFAULTS = {"dtype": None}


class Loop(Stmt):
    FIELDS = ("axis", "body", "seed")
    DEFAULTS = {"body": (), "seed": False}
    TUPLES = ("body",)
    BODIES = ("body",)


class StridedLoop(Stmt):
    FIELDS = ("axis", "start", "step", "body", "end", "seed", "unroll")
    DEFAULTS = {"body": (), "end": None, "seed": False, "unroll": False}
    TUPLES = ("body",)
    BODIES = ("body",)


class Cond(Stmt):
    FIELDS = ("cond", "body", "else_body")
    DEFAULTS = {"body": (), "else_body": ()}
    TUPLES = ("body", "else_body")
    BODIES = ("body", "else_body")


class SelectBranch(Node):
    FIELDS = ("value", "select")


class Select(Stmt):
    FIELDS = ("name", "branches")
    DEFAULTS = {"branches": ()}
    TUPLES = ("branches",)

    def reads(self) -> set[str]:
        out: set[str] = set()
        for br in self.branches:
            if isinstance(br.value, str):
                out.add(br.value)
            if isinstance(br.select, Expr):
                out |= br.select.var_names()
        return out


class Pre(Stmt):
    FIELDS = ("name", "carrier", "index")
    DEFAULTS = {"index": ()}
    TUPLES = ("index",)


class Carry(Stmt):
    FIELDS = ("name", "value", "index", "seed", "dtype")
    DEFAULTS = {"index": (), "seed": 0.0, "dtype": None}
    TUPLES = ("index",)


class ZeroPrologue(Stmt):
    FIELDS = ("dst", "words")


def _opaque(name: str, fields: tuple[str, ...], defaults: dict | None = None) -> type:
    """IR nodes outside the three kernel families (tensor-core fragments, TMA,
    mbarrier, wgmma, cp.async).  They decode so a KernelOp that contains them
    can be reported precisely, but no family lowers them."""
    return type(name, (Stmt,), {"FIELDS": fields, "DEFAULTS": defaults or {}})


CpAsyncCopy = _opaque("CpAsyncCopy", ("smem", "smem_index", "src", "src_index", "nbytes", "lane_index"),
                      {"nbytes": 4, "lane_index": None})
CpAsyncCommit = _opaque("CpAsyncCommit", ())
CpAsyncWait = _opaque("CpAsyncWait", ("group",), {"group": 0})
RegFragment = _opaque("RegFragment", ("name", "role", "shape", "dtype", "nregs"), {"nregs": None})
LdmatrixLoad = _opaque("LdmatrixLoad", ("frag", "src_buffer", "src_index", "role", "b_trans"),
                       {"b_trans": False})
BlockScaleLoad = _opaque("BlockScaleLoad", ("frag", "src_buffer", "src_index", "role"), {"role": "a"})
MmaSyncPtx = _opaque("MmaSyncPtx", ("c_frag", "a_frag", "b_frag", "shape", "ab_dtype", "c_dtype",
                                    "b_row_major"), {"b_row_major": False})
FragmentPromote = _opaque("FragmentPromote", ("dst", "src"))
FragmentApply = _opaque("FragmentApply", ("out", "op", "args", "kinds"), {"args": (), "kinds": ()})
FragmentRowReduce = _opaque("FragmentRowReduce", ("frags", "op", "top", "bot"))
FragmentRepack = _opaque("FragmentRepack", ("frag", "srcs", "ab_dtype"), {"ab_dtype": "f16"})
RegStore = _opaque("RegStore", ("frag", "dst_buffer", "dst_index", "row_base", "col_base", "ldm",
                                "atomic"),
                   {"row_base": None, "col_base": None, "ldm": None, "atomic": False})
TmaDescriptor = _opaque("TmaDescriptor", ("name", "tensor", "global_shape", "box"))
TmaLoad = _opaque("TmaLoad", ("smem", "smem_index", "desc", "coords", "mbar", "mbar_slot"),
                  {"mbar_slot": None})
MbarrierInit = _opaque("MbarrierInit", ("mbar", "count", "slot"), {"slot": None})
MbarrierArrive = _opaque("MbarrierArrive", ("mbar", "slot"), {"slot": None})
MbarrierArriveExpectTx = _opaque("MbarrierArriveExpectTx", ("mbar", "bytes_", "slot"), {"slot": None})
MbarrierWait = _opaque("MbarrierWait", ("mbar", "phase", "slot"), {"slot": None})
SetMaxNReg = _opaque("SetMaxNReg", ("direction", "count"))
WgmmaDescriptor = _opaque("WgmmaDescriptor", ("name", "smem", "smem_index", "swizzle", "lbo_bytes",
                                              "sbo_bytes"),
                          {"smem_index": None, "swizzle": 128, "lbo_bytes": 0, "sbo_bytes": 0})
WgmmaMma = _opaque("WgmmaMma", ("shape", "c_frags", "a_desc", "a_frag", "b_desc", "ab_dtype", "scale_d",
                                "trans_a", "trans_b"),
                   {"a_desc": None, "a_frag": None, "scale_d": 1, "trans_a": 0, "trans_b": 0})
WgmmaFence = _opaque("WgmmaFence", ())
WgmmaCommit = _opaque("WgmmaCommit", ())
WgmmaWait = _opaque("WgmmaWait", ("group",), {"group": 0})


NODE_CLASSES: dict[str, type] = {
    c.__name__: c
    for c in (Dim, DataType, ElementwiseImpl, Tensor, Var, Builtin, Literal, BinaryExpr, TernaryExpr,
              CastExpr, FuncCallExpr, FlatIndex, Axis, KernelOp, Tile, Smem, Sync, WarpShuffle,
              TreeHalve, Load, Write, Assign, Accum, Init, Let, Loop, StridedLoop, Cond, SelectBranch,
              Select, Pre, Carry, ZeroPrologue, CpAsyncCopy, CpAsyncCommit, CpAsyncWait, RegFragment,
              LdmatrixLoad, BlockScaleLoad, MmaSyncPtx, FragmentPromote, FragmentApply,
              FragmentRowReduce, FragmentRepack, RegStore, TmaDescriptor, TmaLoad, MbarrierInit,
              MbarrierArrive, MbarrierArriveExpectTx, MbarrierWait, SetMaxNReg, WgmmaDescriptor,
              WgmmaMma, WgmmaFence, WgmmaCommit, WgmmaWait)
}


# ------------------------------------------------------------------ helpers


def body_stmts(body) -> tuple:
    return () if body is None else tuple(body)


def walk(body):
    """Pre-order walk over statements and their child bodies."""
    for s in body_stmts(body):
        yield s
        for child in s.nested() if isinstance(s, Node) else ():
            yield from walk(child)


def dtype_name(dt) -> str | None:
    if dt is None:
        return None
    if isinstance(dt, str):
        return dt
    return getattr(dt, "name", None) or str(dt)


def op_name(op) -> str:
    return op if isinstance(op, str) else getattr(op, "name", str(op))


F32_NAMES = ("f32", "float", "float32")
F16_NAMES = ("f16", "half", "float16", "__half")
BF16_NAMES = ("bf16", "bfloat16", "__nv_bfloat16")
INT_NAMES = ("i32", "int", "int32", "s32", "u32")


def canon_dtype(dt) -> str:
    """Canonical element type: f32, bf16, f16, i32, f64, u8 ... (default f32)."""
    name = dtype_name(dt)
    if name in (None, ""):
        return "f32"
    if name in F32_NAMES:
        return "f32"
    if name in F16_NAMES:
        return "f16"
    if name in BF16_NAMES:
        return "bf16"
    if name in ("i32", "int", "int32", "s32"):
        return "i32"
    if name == "u32":
        return "u32"
    if name in ("f64", "double"):
        return "f64"
    if name in ("i64", "int64", "s64"):
        return "i64"
    return name


ELEM_BYTES = {"f32": 4, "bf16": 2, "f16": 2, "i32": 4, "u32": 4, "f64": 8, "i64": 8, "u64": 8,
              "u8": 1, "i8": 1}
