"""Minimal stand-in for the Emmy IR data model (``emmy-ml==0.3.11``).

TEST INFRASTRUCTURE ONLY.  The real ``emmy`` package is not installed in this
environment, and the reference compiler (``compile.py`` of
vedantgpt/emmy-ptx-compiler) imports it only to deserialize Kernel IR
(compile.py:42-101).  This module provides the classes, fields and helper
methods that compile.py reads, written from the reference's *usage*:

* constructors as called in tools/make_proxy_set.py:89-365,
  tools/make_world_set.py:68-291 and tests/test_*.py;
* attribute reads in compile.py (e.g. ``s.state_b`` at 2220, ``s.inner`` at
  2247, ``expr.pretty()`` at 1136, ``expr.simplify(ctx)`` at 2644-2648,
  ``stmt.nested()`` at 256, ``stmt.deps()`` at 1416).

Every node's ``repr`` is eval-round-trippable, because the IR JSON stores the
kernel body as ``repr(body)`` (tools/make_proxy_set.py:49-55) and
``Graph.from_dict`` evaluates it back.  Only tests/ and the golden-fixture
generator put this directory on ``sys.path``; the product never imports it.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Any

import numpy as np


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
    if isinstance(v, list):
        return "[" + ", ".join(_fmt(x) for x in v) + "]"
    if isinstance(v, dict):
        return "{" + ", ".join(f"{_fmt(k)}: {_fmt(x)}" for k, x in v.items()) + "}"
    return repr(v)


class _Node:
    """Dataclass-style repr with keyword fields (eval-round-trippable)."""

    _fields: tuple[str, ...] = ()

    def __repr__(self) -> str:
        parts = ", ".join(f"{f}={_fmt(getattr(self, f))}" for f in self._fields)
        return f"{type(self).__name__}({parts})"

    def __eq__(self, other: object) -> bool:
        return type(self) is type(other) and all(
            getattr(self, f) == getattr(other, f) for f in self._fields
        )

    def __hash__(self) -> int:
        return hash((type(self).__name__, repr(self)))


def _tup(x) -> tuple:
    if x is None:
        return ()
    if isinstance(x, (list, tuple)):
        return tuple(x)
    return (x,)


# --------------------------------------------------------------------------- dims


class Dim(_Node):
    """Static extent.  ``repr`` is ``Dim(64)`` (tools/make_proxy_set.py:398-399
    rewrites bodies by replacing that exact text)."""

    _fields = ("value",)

    def __init__(self, value):
        self.value = int(value)

    def as_static(self) -> int:
        return self.value

    def __int__(self) -> int:
        return self.value

    def __repr__(self) -> str:
        return f"Dim({self.value})"


class Tensor(_Node):
    _fields = ("name", "shape", "dtype")

    def __init__(self, name, shape=(), dtype="f32"):
        self.name = name
        self.shape = tuple(shape)
        self.dtype = dtype


class InputOp(_Node):
    _fields = ("name",)

    def __init__(self, name=""):
        self.name = name


class ConstantOp(_Node):
    _fields = ("name", "value")

    def __init__(self, name="", value=None, **_):
        self.name = name
        self.value = value


class ElementwiseImpl(_Node):
    _fields = ("name", "identity")

    def __init__(self, name, identity=None):
        self.name = name
        self.identity = identity


class DataType(_Node):
    _fields = ("name", "np_dtype", "itemsize")

    def __init__(self, name, np_dtype=None, itemsize=4):
        self.name = name
        self.np_dtype = np.dtype(np_dtype) if np_dtype is not None else None
        self.itemsize = int(itemsize)

    def __str__(self) -> str:
        return self.name


# --------------------------------------------------------------------------- exprs


class SimplifyCtx:
    @staticmethod
    def empty() -> "SimplifyCtx":
        return SimplifyCtx()


class _Expr(_Node):
    def simplify(self, ctx=None):
        return self

    def vars(self) -> set[str]:
        out: set[str] = set()
        for f in self._fields:
            v = getattr(self, f)
            for item in (v if isinstance(v, tuple) else (v,)):
                if isinstance(item, _Expr):
                    out |= item.vars()
        return out


class Var(_Expr):
    _fields = ("name",)

    def __init__(self, name):
        self.name = name

    def pretty(self) -> str:
        return self.name

    def vars(self) -> set[str]:
        return {self.name}


class Builtin(_Expr):
    _fields = ("name",)

    def __init__(self, name):
        self.name = name

    def pretty(self) -> str:
        return self.name


class Literal(_Expr):
    _fields = ("value", "dtype")

    def __init__(self, value, dtype=None):
        self.value = value
        self.dtype = dtype

    def pretty(self) -> str:
        return repr(self.value)


class BinaryExpr(_Expr):
    _fields = ("op", "left", "right")

    def __init__(self, op, left, right):
        self.op = op
        self.left = left
        self.right = right

    def pretty(self) -> str:
        return f"({self.left.pretty()} {self.op} {self.right.pretty()})"


class TernaryExpr(_Expr):
    _fields = ("cond", "if_true", "if_false")

    def __init__(self, cond, if_true, if_false):
        self.cond = cond
        self.if_true = if_true
        self.if_false = if_false

    def pretty(self) -> str:
        return f"({self.cond.pretty()} ? {self.if_true.pretty()} : {self.if_false.pretty()})"


class CastExpr(_Expr):
    """compile.py reads both ``.expr`` (2690) and ``.value`` (697)."""

    _fields = ("expr", "dtype")

    def __init__(self, expr, dtype):
        self.expr = expr
        self.dtype = dtype

    @property
    def value(self):
        return self.expr

    def pretty(self) -> str:
        return f"(({self.dtype}){self.expr.pretty()})"


class FuncCallExpr(_Expr):
    _fields = ("name", "args")

    def __init__(self, name, args=()):
        self.name = name
        self.args = _tup(args)

    def pretty(self) -> str:
        return f"{self.name}(" + ", ".join(a.pretty() for a in self.args) + ")"


class FlatIndex(_Expr):
    _fields = ("buffer", "index")

    def __init__(self, buffer, index=()):
        self.buffer = buffer
        self.index = _tup(index)

    def pretty(self) -> str:
        return f"flat({self.buffer}[" + ", ".join(i.pretty() for i in self.index) + "])"


# --------------------------------------------------------------------------- stmts


class _Stmt(_Node):
    _bodies: tuple[str, ...] = ()

    def nested(self):
        return tuple(getattr(self, b) for b in self._bodies)

    def deps(self) -> set[str]:
        out: set[str] = set()
        for f in self._fields:
            if f in self._bodies:
                continue
            v = getattr(self, f)
            for item in (v if isinstance(v, tuple) else (v,)):
                if isinstance(item, _Expr):
                    out |= item.vars()
        return out


class Axis(_Node):
    _fields = ("name", "extent")

    def __init__(self, name, extent):
        self.name = name
        self.extent = extent if isinstance(extent, Dim) else Dim(int(extent))


class KernelOp(_Node):
    _fields = ("name", "body", "inputs", "outputs")

    def __init__(self, name, body=(), inputs=None, outputs=None):
        self.name = name
        self.body = _tup(body)
        self.inputs = dict(inputs or {})
        self.outputs = dict(outputs or {})


class Tile(_Stmt):
    _fields = ("axes", "body", "block_threads", "aux_threads", "raster_group",
               "raster_axes", "raster_orient")
    _bodies = ("body",)

    def __init__(self, axes, body=(), block_threads=None, aux_threads=0, raster_group=None,
                 raster_axes=None, raster_orient=None):
        self.axes = _tup(axes)
        self.body = _tup(body)
        self.block_threads = block_threads
        self.aux_threads = aux_threads
        self.raster_group = raster_group
        self.raster_axes = raster_axes
        self.raster_orient = raster_orient


class Smem(_Stmt):
    _fields = ("name", "extents", "dtype", "align")

    def __init__(self, name, extents, dtype="f32", align=0):
        self.name = name
        self.extents = _tup(extents)
        self.dtype = dtype
        self.align = align


class Sync(_Stmt):
    _fields = ("barrier_id", "count", "warp")

    def __init__(self, barrier_id=0, count=0, warp=False):
        self.barrier_id = barrier_id
        self.count = count
        self.warp = warp


class WarpShuffle(_Stmt):
    _fields = ("state", "state_b", "combine_states", "length", "dtype")

    def __init__(self, state, state_b, combine_states, length=32, dtype=None):
        self.state = _tup(state)
        self.state_b = _tup(state_b)
        self.combine_states = _tup(combine_states)
        self.length = length
        self.dtype = dtype

    def deps(self) -> set[str]:
        return set(self.state)


class TreeHalve(_Stmt):
    _fields = ("bufs", "state", "state_b", "combine_states", "length", "tid_var", "inner",
               "barrier_id", "barrier_count", "dtype")

    def __init__(self, bufs, state, state_b, combine_states, length, tid_var, inner=None,
                 barrier_id=0, barrier_count=0, dtype=None):
        self.bufs = _tup(bufs)
        self.state = _tup(state)
        self.state_b = _tup(state_b)
        self.combine_states = _tup(combine_states)
        self.length = length
        self.tid_var = tid_var
        self.inner = inner
        self.barrier_id = barrier_id
        self.barrier_count = barrier_count
        self.dtype = dtype

    def deps(self) -> set[str]:
        return set(self.state) | {self.tid_var}


class Load(_Stmt):
    _fields = ("names", "input", "index", "dtype")

    def __init__(self, names, input, index=(), dtype=None):
        self.names = _tup(names)
        self.input = input
        self.index = _tup(index)
        self.dtype = dtype


class Write(_Stmt):
    _fields = ("output", "index", "values", "value_dtype", "atomic")

    def __init__(self, output, index=(), values=(), value_dtype=None, atomic=False):
        self.output = output
        self.index = _tup(index)
        self.values = _tup(values)
        self.value_dtype = value_dtype
        self.atomic = atomic

    def deps(self) -> set[str]:
        return super().deps() | set(self.values)


class Assign(_Stmt):
    _fields = ("name", "op", "args", "dtype")

    def __init__(self, name, op, args=(), dtype=None):
        self.name = name
        self.op = op
        self.args = _tup(args)
        self.dtype = dtype

    def deps(self) -> set[str]:
        return set(a for a in self.args if isinstance(a, str))


class Accum(_Stmt):
    _fields = ("name", "value", "op", "dtype", "axes", "base")

    def __init__(self, name, value, op=None, dtype=None, axes=(), base=None):
        self.name = name
        self.value = value
        self.op = op if op is not None else ElementwiseImpl("add")
        self.dtype = dtype
        self.axes = _tup(axes)
        self.base = base

    def deps(self) -> set[str]:
        return {x for x in (self.value, self.base) if isinstance(x, str)}


class Init(_Stmt):
    _fields = ("name", "identity", "dtype")

    def __init__(self, name, identity=0.0, dtype=None):
        self.name = name
        self.identity = identity
        self.dtype = dtype


class Let(_Stmt):
    _fields = ("name", "value", "dtype")

    def __init__(self, name, value, dtype=None):
        self.name = name
        self.value = value
        self.dtype = dtype


class Loop(_Stmt):
    _fields = ("axis", "body", "seed")
    _bodies = ("body",)

    def __init__(self, axis, body=(), seed=False):
        self.axis = axis
        self.body = _tup(body)
        self.seed = seed


class StridedLoop(_Stmt):
    _fields = ("axis", "start", "step", "body", "end", "seed", "unroll")
    _bodies = ("body",)

    def __init__(self, axis, start, step, body=(), end=None, seed=False, unroll=False):
        self.axis = axis
        self.start = start
        self.step = step
        self.body = _tup(body)
        self.end = end
        self.seed = seed
        self.unroll = unroll


class Cond(_Stmt):
    _fields = ("cond", "body", "else_body")
    _bodies = ("body", "else_body")

    def __init__(self, cond, body=(), else_body=()):
        self.cond = cond
        self.body = _tup(body)
        self.else_body = _tup(else_body)


class Pre(_Stmt):
    _fields = ("name", "carrier", "index")

    def __init__(self, name, carrier, index=()):
        self.name = name
        self.carrier = carrier
        self.index = _tup(index)


class Carry(_Stmt):
    _fields = ("name", "value", "index", "seed", "dtype")

    def __init__(self, name, value, index=(), seed=0.0, dtype=None):
        self.name = name
        self.value = value
        self.index = _tup(index)
        self.seed = seed
        self.dtype = dtype


class ZeroPrologue(_Stmt):
    _fields = ("dst", "words")

    def __init__(self, dst, words):
        self.dst = dst
        self.words = words


class SelectBranch(_Node):
    _fields = ("value", "select")

    def __init__(self, value, select):
        self.value = value
        self.select = select


class Select(_Stmt):
    _fields = ("name", "branches")

    def __init__(self, name, branches=()):
        self.name = name
        self.branches = _tup(branches)

    def deps(self) -> set[str]:
        out: set[str] = set()
        for br in self.branches:
            if isinstance(br.value, str):
                out.add(br.value)
            if isinstance(br.select, _Expr):
                out |= br.select.vars()
        return out


# ------------------------------------------------- extra-ISA nodes (compile.py:2938-3161)


def _simple(name: str, fields: tuple[str, ...], defaults: dict | None = None):
    defaults = defaults or {}

    def __init__(self, *args, **kwargs):
        if len(args) > len(fields):
            raise TypeError(f"{name}: too many positional arguments")
        vals = dict(zip(fields, args))
        for k, v in kwargs.items():
            if k not in fields:
                raise TypeError(f"{name}: unexpected field {k!r}")
            vals[k] = v
        for f in fields:
            if f in vals:
                setattr(self, f, vals[f])
            elif f in defaults:
                setattr(self, f, defaults[f])
            else:
                raise TypeError(f"{name}: missing field {f!r}")

    return type(name, (_Stmt,), {"_fields": fields, "__init__": __init__})


CpAsyncCopy = _simple("CpAsyncCopy", ("smem", "smem_index", "src", "src_index", "nbytes", "lane_index"),
                      {"lane_index": None, "nbytes": 4})
CpAsyncCommit = _simple("CpAsyncCommit", ())
CpAsyncWait = _simple("CpAsyncWait", ("group",), {"group": 0})
RegFragment = _simple("RegFragment", ("name", "role", "shape", "dtype", "nregs"), {"nregs": None})
LdmatrixLoad = _simple("LdmatrixLoad", ("frag", "src_buffer", "src_index", "role", "b_trans"),
                       {"b_trans": False})
BlockScaleLoad = _simple("BlockScaleLoad", ("frag", "src_buffer", "src_index", "role"), {"role": "a"})
MmaSyncPtx = _simple("MmaSyncPtx", ("c_frag", "a_frag", "b_frag", "shape", "ab_dtype", "c_dtype",
                                    "b_row_major"), {"b_row_major": False})
FragmentPromote = _simple("FragmentPromote", ("dst", "src"))
FragmentApply = _simple("FragmentApply", ("out", "op", "args", "kinds"), {"args": (), "kinds": ()})
FragmentRowReduce = _simple("FragmentRowReduce", ("frags", "op", "top", "bot"))
FragmentRepack = _simple("FragmentRepack", ("frag", "srcs", "ab_dtype"), {"ab_dtype": "f16"})
RegStore = _simple("RegStore", ("frag", "dst_buffer", "dst_index", "row_base", "col_base", "ldm",
                                "atomic"),
                   {"row_base": None, "col_base": None, "ldm": None, "atomic": False})
TmaDescriptor = _simple("TmaDescriptor", ("name", "tensor", "global_shape", "box"))
TmaLoad = _simple("TmaLoad", ("smem", "smem_index", "desc", "coords", "mbar", "mbar_slot"),
                  {"mbar_slot": None})
MbarrierInit = _simple("MbarrierInit", ("mbar", "count", "slot"), {"slot": None})
MbarrierArrive = _simple("MbarrierArrive", ("mbar", "slot"), {"slot": None})
MbarrierArriveExpectTx = _simple("MbarrierArriveExpectTx", ("mbar", "bytes_", "slot"), {"slot": None})
MbarrierWait = _simple("MbarrierWait", ("mbar", "phase", "slot"), {"slot": None})
SetMaxNReg = _simple("SetMaxNReg", ("direction", "count"))
WgmmaDescriptor = _simple("WgmmaDescriptor", ("name", "smem", "smem_index", "swizzle", "lbo_bytes",
                                              "sbo_bytes"),
                          {"smem_index": None, "swizzle": 128, "lbo_bytes": 0, "sbo_bytes": 0})
WgmmaMma = _simple("WgmmaMma", ("shape", "c_frags", "a_desc", "a_frag", "b_desc", "ab_dtype", "scale_d",
                                "trans_a", "trans_b"),
                   {"a_desc": None, "a_frag": None, "scale_d": 1, "trans_a": 0, "trans_b": 0})
WgmmaFence = _simple("WgmmaFence", ())
WgmmaCommit = _simple("WgmmaCommit", ())
WgmmaWait = _simple("WgmmaWait", ("group",), {"group": 0})


# --------------------------------------------------------------------------- graph


def _namespace() -> dict:
    ns = {k: v for k, v in globals().items() if isinstance(v, type)}
    ns["dtype"] = np.dtype
    ns["float"] = float
    ns["__builtins__"] = {}
    return ns


def decode_body(text: str):
    """Evaluate one ``repr(body)`` string back into shim nodes."""
    return eval(text, _namespace())  # noqa: S307 - fixtures are produced by this shim


class Node:
    def __init__(self, name: str, op, inputs=(), outputs=()):
        self.name = name
        self.op = op
        self.inputs = list(inputs)
        self.outputs = list(outputs)


class Graph:
    def __init__(self, inputs, outputs, nodes: dict[str, Node]):
        self.inputs = list(inputs)
        self.outputs = list(outputs)
        self.nodes = nodes

    @classmethod
    def from_dict(cls, raw: dict) -> "Graph":
        out_tensors: dict[str, Tensor] = {}
        for name, nd in raw.get("nodes", {}).items():
            for o in nd.get("outputs") or []:
                out_tensors[o["name"]] = Tensor(o["name"], tuple(Dim(x) for x in o.get("shape") or ()),
                                                o.get("dtype") or "f32")
        nodes: dict[str, Node] = {}
        for name, nd in raw.get("nodes", {}).items():
            kind = nd.get("op")
            fields = nd.get("op_fields") or {}
            if kind == "KernelOp":
                body = []
                for text in fields.get("body") or []:
                    b = decode_body(text)
                    body.extend(b if isinstance(b, (tuple, list)) else (b,))
                ins = {i: out_tensors.get(i, Tensor(i)) for i in nd.get("inputs") or []}
                outs = {o["name"]: out_tensors[o["name"]] for o in nd.get("outputs") or []}
                op = KernelOp(fields.get("name", name), tuple(body), ins, outs)
            elif kind == "ConstantOp":
                op = ConstantOp(fields.get("name", name), fields.get("value"))
            else:
                op = InputOp(name)
            nodes[name] = Node(name, op, nd.get("inputs") or [], nd.get("outputs") or [])
        return cls(raw.get("inputs") or [], raw.get("outputs") or [], nodes)
