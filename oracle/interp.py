"""CPU oracle: evaluate an Emmy KernelOp the way the reference compiler's PTX does.

TEST INFRASTRUCTURE ONLY.  Imported by tests/, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU baseline / reference arm - never by the product.

The IR is decoded with the test shim (``oracle/emmy_shim``).  Semantics
restated from vedantgpt/emmy-ptx-compiler's compile.py:

* per-cell statement walk with the two FMA lookahead rules
  (``stmts``/``_try_fma``/``_try_fma_assign``, compile.py:1096-1131,
  1263-1303, ``_uses_name`` 1415-1428);
* the Assign op table (compile.py:2068-2199) - IEEE f32 ops through numpy's
  float32 ufuncs (correctly rounded, like ``add/sub/mul/div.rn/sqrt.rn/rcp.rn``),
  ``max/min.f32`` as ``fmax/fmin``, ordered compares, and the
  approximate ``ex2/lg2/rsqrt`` through ``oracle/oracle.c``;
* ``Let`` literals rounded to f32 (compile.py:1942-1952, ``f32_hex`` 205-207),
  accumulator identities (compile.py:327-338), Select (2915-2936), Cond
  (1916-1933), index flattening (2466-2493);
* reductions in the reference schedule's exact order (strided per-thread
  accumulation, 5-step butterfly, smem tree: compile.py:1866-1914,
  2213-2286) via ``ora_strided_reduce_f32``, the one-thread-per-row Loop
  (1813-1864) via ``ora_loop_reduce_f32``, and the naive matmul's sequential
  FMA over k via ``ora_gemm_seqfma_f32``.

Vectorised over all Tile cells with numpy; meant for sizes up to a few
hundred million element-ops.
"""

from __future__ import annotations

import ctypes as C
import json
import math
import subprocess
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE / "emmy_shim"))

from emmy._core import (  # noqa: E402
    Accum, Assign, BinaryExpr, Builtin, CastExpr, Cond, FlatIndex, FuncCallExpr, Graph, Init, KernelOp,
    Let, Literal, Load, Loop, Select, Smem, StridedLoop, Sync, TernaryExpr, Tile, TreeHalve, Var, ZeroPrologue,
    WarpShuffle, Write, CpAsyncCopy, CpAsyncCommit, CpAsyncWait, Pre, Carry,
)

_LIB = None


def lib():
    global _LIB
    if _LIB is None:
        so = HERE / "build" / "liboracle.so"
        if not so.is_file() or so.stat().st_mtime < (HERE / "oracle.c").stat().st_mtime:
            subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
        L = C.CDLL(str(so))
        fp, vp, i64, i32, f32 = C.POINTER(C.c_float), C.c_void_p, C.c_int64, C.c_int, C.c_float
        L.ora_fma_f32.argtypes = [vp, vp, vp, vp, C.c_size_t]
        for n in ("ora_ex2_f32", "ora_lg2_f32", "ora_rsqrt_f32"):
            getattr(L, n).argtypes = [vp, vp, C.c_size_t]
        L.ora_gemm_seqfma_f32.argtypes = [vp, vp, vp, i64, i64, i64, i32]
        L.ora_strided_reduce_f32.argtypes = [vp, vp, i64, i64, i32, i32, f32, vp]
        L.ora_loop_reduce_f32.argtypes = [vp, vp, i64, i64, i32, f32, vp]
        L.ora_row_sum_f64.argtypes = [vp, i64, i64, vp]
        L.ora_attn_naive_f32.argtypes = [vp, vp, vp, vp, i64, i64, i64, i64, f32]
        L.ora_attn_naive_f32.restype = i32
        del fp
        _LIB = L
    return _LIB


def _p(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def c_fma(a, b, c) -> np.ndarray:
    a, b, c = np.broadcast_arrays(*(np.asarray(v, np.float32) for v in (a, b, c)))
    a, b, c = (np.ascontiguousarray(v) for v in (a, b, c))
    out = np.empty(a.shape, np.float32)
    lib().ora_fma_f32(_p(a), _p(b), _p(c), _p(out), out.size)
    return out


def _c_unary(name: str, x) -> np.ndarray:
    x = np.ascontiguousarray(np.asarray(x, np.float32))
    out = np.empty(x.shape, np.float32)
    getattr(lib(), name)(_p(x), _p(out), out.size)
    return out


def ex2(x):
    return _c_unary("ora_ex2_f32", x)


def lg2(x):
    return _c_unary("ora_lg2_f32", x)


def rsqrt(x):
    return _c_unary("ora_rsqrt_f32", x)


F32 = np.float32
LOG2E = F32(1.0 / math.log(2.0))
LN2 = F32(math.log(2.0))
IDENT = {"add": 0.0, "sum": 0.0, "multiply": 1.0, "prod": 1.0, "maximum": -1e30, "amax": -1e30,
         "max": -1e30, "minimum": 1e30, "min": 1e30}
F32_NAMES = ("f32", "float", "float32")


def opname(op) -> str:
    return op if isinstance(op, str) else getattr(op, "name", str(op))


def dtname(dt) -> str | None:
    if dt is None:
        return None
    return dt if isinstance(dt, str) else getattr(dt, "name", str(dt))


def identity_of(op) -> float:
    ident = getattr(op, "identity", None) if not isinstance(op, str) else None
    if ident is not None:
        return float(ident)
    return IDENT.get(opname(op), 0.0)


def combine(op: str, a, b):
    a, b = np.asarray(a, F32), np.asarray(b, F32)
    if op in ("maximum", "amax", "max"):
        return np.fmax(a, b)
    if op in ("minimum", "amin", "min"):
        return np.fmin(a, b)
    if op in ("multiply", "mul", "prod"):
        return np.multiply(a, b, dtype=F32)
    if op in ("subtract", "sub"):
        return np.subtract(a, b, dtype=F32)
    if op in ("divide", "true_divide", "div"):
        return np.divide(a, b, dtype=F32)
    return np.add(a, b, dtype=F32)


def ordered_cmp(op: str, a, b):
    a, b = np.asarray(a), np.asarray(b)
    with np.errstate(invalid="ignore"):
        if op == "!=":
            return (a < b) | (a > b)
        return {"<": np.less, "<=": np.less_equal, ">": np.greater, ">=": np.greater_equal,
                "==": np.equal}[op](a, b)


CMP = {"gt": ">", "greater": ">", "lt": "<", "less": "<", "ge": ">=", "greater_equal": ">=",
       "le": "<=", "less_equal": "<=", "eq": "==", "equal": "==", "ne": "!=", "not_equal": "!="}


def f32_op(op: str, args: list):
    """compile.py:2087-2199 on f32 operands."""
    a = [np.asarray(x, F32) for x in args]
    with np.errstate(all="ignore"):
        if op in ("add", "sum", "subtract", "sub", "multiply", "mul", "divide", "true_divide", "div",
                  "maximum", "amax", "max", "minimum", "amin", "min") and len(a) == 2:
            return combine(op, a[0], a[1])
        if op in CMP and len(a) == 2:
            return np.where(ordered_cmp(CMP[op], a[0], a[1]), F32(1), F32(0))
        if op == "exp2":
            return ex2(a[0])
        if op in ("exp", "exp_fast"):
            return ex2(np.multiply(a[0], LOG2E, dtype=F32))
        if op == "sqrt":
            return np.sqrt(a[0], dtype=F32)
        if op == "rsqrt":
            return rsqrt(a[0])
        if op in ("reciprocal", "recip"):
            return np.divide(F32(1), a[0], dtype=F32)
        if op == "square":
            return np.multiply(a[0], a[0], dtype=F32)
        if op in ("clamp", "clip") and len(a) == 3:
            return np.fmin(np.fmax(a[0], a[1]), a[2])
        if op == "relu":
            return np.fmax(a[0], F32(0))
        if op == "leaky_relu":
            slope = a[1] if len(a) > 1 else F32(0.01)
            return np.where(ordered_cmp(">", a[0], F32(0)), a[0], np.multiply(a[0], slope, dtype=F32))
        if op in ("neg", "negative"):
            return np.negative(a[0])
        if op in ("abs", "absolute"):
            return np.abs(a[0])
        if op == "copy":
            return a[0].copy()
        if op in ("log", "log_fast"):
            return np.multiply(lg2(a[0]), LN2, dtype=F32)
        if op in ("log2", "lg2"):
            return lg2(a[0])
        if op == "tanh":
            two_x = np.multiply(a[0], F32(2), dtype=F32)
            e = ex2(np.multiply(two_x, LOG2E, dtype=F32))
            return np.divide(np.subtract(e, F32(1), dtype=F32), np.add(e, F32(1), dtype=F32), dtype=F32)
        if op in ("sigmoid", "silu"):
            e = ex2(np.multiply(np.negative(a[0]), LOG2E, dtype=F32))
            sig = np.divide(F32(1), np.add(F32(1), e, dtype=F32), dtype=F32)
            return sig if op == "sigmoid" else np.multiply(a[0], sig, dtype=F32)
        if op == "pow" and len(a) == 2:
            return ex2(np.multiply(lg2(a[0]), a[1], dtype=F32))
    raise NotImplementedError(f"oracle: op {op!r}")


def bf16_round(x: np.ndarray) -> np.ndarray:
    """cvt.rn.bf16.f32: round-to-nearest-even to bf16, returned as float32."""
    x = np.ascontiguousarray(x, F32)
    bits = x.view(np.uint32).astype(np.uint64)
    rnd = ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16) << 16
    out = rnd.astype(np.uint32).view(F32).copy()
    nan = np.isnan(x)
    out[nan] = np.nan
    return out


def f16_round(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, F32).astype(np.float16).astype(F32)


def store_cast(vals: np.ndarray, dt: str | None) -> np.ndarray:
    if dt in (None, *F32_NAMES):
        return np.asarray(vals, F32)
    if dt == "bf16":
        return bf16_round(vals)
    if dt in ("f16", "half", "float16"):
        return f16_round(vals)
    if dt in ("i32", "int", "int32", "s32"):
        return np.trunc(np.asarray(vals, F32)).astype(np.float32)
    raise NotImplementedError(dt)


def uses_name(stmt, name: str) -> bool:
    if hasattr(stmt, "deps") and name in stmt.deps():
        return True
    if isinstance(stmt, Write) and name in stmt.values:
        return True
    if isinstance(stmt, Assign) and name in stmt.args:
        return True
    if isinstance(stmt, Accum) and name in (stmt.value, stmt.base):
        return True
    for child in stmt.nested():
        for t in child:
            if uses_name(t, name):
                return True
    return False


def row_major(shape) -> list[int]:
    st = [1] * len(shape)
    acc = 1
    for d in range(len(shape) - 1, -1, -1):
        st[d] = acc
        acc *= int(shape[d])
    return st


# ------------------------------------------------------------------ cell machine


class Cells:
    """Evaluate straight-line IR over N cells at once (vectorised lanes)."""

    def __init__(self, n: int, bufs: dict[str, np.ndarray], shapes: dict, dtypes: dict):
        self.n = n
        self.bufs = bufs      # flat float32 arrays (inputs + outputs)
        self.shapes = shapes
        self.dtypes = dtypes
        self.env: dict[str, tuple[str, np.ndarray]] = {}
        self.mask: np.ndarray | None = None
        # plain mul.f32 results the assembler may fuse into a following add/sub
        self.products: dict[str, tuple] = {}
        self.fusable: set | None = None
        self.order = 0

    # values -----------------------------------------------------------------
    def f32(self, name):
        if isinstance(name, str) and name in self.env:
            k, v = self.env[name]
            if k == "f32":
                return v
            if k == "int":
                return np.asarray(v).astype(F32)
            return np.where(v, F32(1), F32(0))
        return F32(float(name))

    def pred(self, name):
        if isinstance(name, str) and name in self.env and self.env[name][0] == "pred":
            return self.env[name][1]
        return ordered_cmp("!=", self.f32(name), F32(0))

    def bind(self, name: str, kind: str, val) -> None:
        self.products.pop(name, None)
        val = np.asarray(val)
        if self.mask is not None and name in self.env:
            ok, old = self.env[name]
            if ok == kind:
                val = np.where(self.mask, val, old)
        elif self.mask is not None:
            zero = F32(0) if kind == "f32" else (0 if kind == "int" else False)
            val = np.where(self.mask, val, zero)
        self.env[name] = (kind, val)

    def expr(self, e):
        if isinstance(e, Literal):
            v = e.value
            if isinstance(v, bool):
                return "int", np.int64(int(v))
            if e.dtype in ("int", "i32", "s32") or (isinstance(v, int) and e.dtype != "float"):
                return "int", np.int64(int(v))
            return "f32", F32(float(v))
        if isinstance(e, Var):
            if e.name in self.env:
                return self.env[e.name]
            raise KeyError(f"oracle: unbound var {e.name}")
        if isinstance(e, Builtin):
            raise NotImplementedError("oracle: thread builtins")
        if isinstance(e, CastExpr):
            k, v = self.expr(e.expr)
            if dtname(e.dtype) in F32_NAMES:
                return "f32", self._tof(k, v)
            return "int", self._toi(k, v)
        if isinstance(e, TernaryExpr):
            p = self._top(*self.expr(e.cond))
            tk, tv = self.expr(e.if_true)
            fk, fv = self.expr(e.if_false)
            if "f32" in (tk, fk):
                return "f32", np.where(p, self._tof(tk, tv), self._tof(fk, fv)).astype(F32)
            return "int", np.where(p, self._toi(tk, tv), self._toi(fk, fv))
        if isinstance(e, FuncCallExpr):
            return "f32", f32_op(e.name, [self._tof(*self.expr(a)) for a in e.args])
        if isinstance(e, FlatIndex):
            return "int", self.flat(e.buffer, e.index)
        if isinstance(e, BinaryExpr):
            return self.binary(e)
        raise NotImplementedError(type(e).__name__)

    @staticmethod
    def _tof(k, v):
        if k == "f32":
            return np.asarray(v, F32)
        if k == "int":
            return np.asarray(v).astype(F32)
        return np.where(v, F32(1), F32(0))

    @staticmethod
    def _toi(k, v):
        if k == "int":
            return np.asarray(v, np.int64)
        if k == "f32":
            with np.errstate(invalid="ignore"):
                return np.trunc(np.asarray(v, F32)).astype(np.int64)
        return np.asarray(v).astype(np.int64)

    def _top(self, k, v):
        if k == "pred":
            return np.asarray(v, bool)
        if k == "f32":
            return ordered_cmp("!=", v, F32(0))
        return np.asarray(v) != 0

    def binary(self, e):
        op = e.op
        if op in ("&&", "||"):
            a, b = self._top(*self.expr(e.left)), self._top(*self.expr(e.right))
            return "pred", (a & b) if op == "&&" else (a | b)
        lk, lv = self.expr(e.left)
        rk, rv = self.expr(e.right)
        if op in ("<", "<=", ">", ">=", "==", "!="):
            if "f32" in (lk, rk):
                return "pred", ordered_cmp(op, self._tof(lk, lv), self._tof(rk, rv))
            return "pred", ordered_cmp(op, self._toi(lk, lv), self._toi(rk, rv))
        if "f32" in (lk, rk):
            a, b = self._tof(lk, lv), self._tof(rk, rv)
            f = {"+": "add", "-": "subtract", "*": "multiply", "/": "divide", "//": "divide"}[op]
            return "f32", combine(f, a, b)
        a, b = self._toi(lk, lv), self._toi(rk, rv)
        if op == "+":
            return "int", a + b
        if op == "-":
            return "int", a - b
        if op == "*":
            return "int", a * b
        if op in ("/", "//"):
            return "int", np.trunc(a / b).astype(np.int64)
        if op == "%":
            return "int", np.fmod(a, b)
        if op == "^":
            return "int", a ^ b
        if op == "&":
            return "int", a & b
        if op == "|":
            return "int", a | b
        if op in ("<<", "shl"):
            return "int", a << b
        if op in (">>", "shr"):
            return "int", a >> b
        raise NotImplementedError(op)

    def flat(self, buf: str, indices):
        indices = tuple(indices)
        if not indices:
            return np.int64(0)
        shape = self.shapes.get(buf)
        if len(indices) == 1:
            return self._toi(*self.expr(indices[0]))
        if not shape or len(shape) != len(indices):
            acc = np.int64(0)
            for ix in indices:
                acc = acc + self._toi(*self.expr(ix))
            return acc
        acc = np.int64(0)
        for ix, st in zip(indices, row_major(shape)):
            acc = acc + self._toi(*self.expr(ix)) * st
        return acc

    def idx_plus(self, indices, k: int):
        if k == 0:
            return tuple(indices)
        return tuple(indices[:-1]) + (BinaryExpr("+", indices[-1], Literal(k, "int")),)

    # statements -------------------------------------------------------------
    def count_uses(self, body) -> None:
        """Find the plain products ptxas folds into FMAs: defined once by a
        multiply/square/log/silu Assign (a plain mul.f32 in the reference's PTX)
        and read only as an operand of plain add/sub Assigns or add Accums."""
        def walk(b):
            for t in b:
                yield t
                for child in t.nested():
                    yield from walk(child)
        defs: dict = {}
        for t in walk(body):
            names = list(t.names) if isinstance(t, Load) else (
                [t.name] if isinstance(t, (Assign, Let, Init, Select)) else [])
            for n in names:
                defs[n] = defs.get(n, 0) + 1
        cands = {t.name for t in walk(body) if isinstance(t, Assign)
                 and opname(t.op) in ("multiply", "mul", "square", "log", "log_fast", "silu") and defs.get(t.name) == 1}
        # Carry / Pre are plain moves the assembler sees through (compile.py:2868-2888)
        alias: dict = {}
        carried: dict = {}
        for t in walk(body):
            if isinstance(t, Carry) and isinstance(t.value, str):
                carried[(t.name, _slot_of(t.index))] = t.value
                alias[t.name] = t.value
            elif isinstance(t, Pre):
                src = carried.get((t.carrier, _slot_of(t.index))) or carried.get((t.carrier, "_"))
                if src is not None:
                    alias[t.name] = src

        def root(n):
            for _ in range(len(alias) + 1):
                if n not in alias:
                    break
                n = alias[n]
            return n
        bad = set()
        for t in walk(body):
            if isinstance(t, Carry):
                continue
            fusing: set = set()
            if isinstance(t, Assign) and opname(t.op) in ("add", "sum", "subtract", "sub") and len(t.args) == 2:
                fusing = {a for a in t.args if isinstance(a, str)}
            elif isinstance(t, Accum) and opname(t.op) in ("add", "sum") and t.base in (None, t.name):
                fusing = {t.value}
            reads: list = []
            if isinstance(t, Assign):
                reads = [a for a in t.args if isinstance(a, str)]
            elif isinstance(t, Accum):
                reads = [x for x in (t.value, t.base) if isinstance(x, str)]
            elif isinstance(t, Write):
                reads = [v for v in t.values if isinstance(v, str)] + sorted(
                    set().union(*[ix.vars() for ix in t.index]) if t.index else set())
            elif isinstance(t, (Select, Load, Let, Cond)):
                reads = sorted(t.deps())
            for n in reads:
                r = root(n) if isinstance(n, str) else n
                if r in cands and n not in fusing:
                    bad.add(r)
        ok = cands - bad
        self.fusable = ok | {n for n in alias if root(n) in ok}

    def product(self, name):
        """Factors of a plain product ptxas folds into the current add/sub
        (pinned by the p_contract_* golden vectors captured on B200)."""
        if isinstance(name, str) and name in self.products and self.fusable is not None and name in self.fusable:
            return self.products[name]
        return None

    def run(self, body) -> None:
        if self.fusable is None:
            self.count_uses(body)
        sl = list(body)
        i = 0
        while i < len(sl):
            s = sl[i]
            nxt = sl[i + 1] if i + 1 < len(sl) else None
            rest = sl[i + 2:]
            if self._fma_accum(s, nxt, rest) or self._fma_assign(s, nxt, rest):
                i += 2
                continue
            self.stmt(s)
            i += 1

    def _fma_accum(self, s, nxt, rest) -> bool:
        if not (isinstance(s, Assign) and isinstance(nxt, Accum)):
            return False
        if opname(s.op) != "multiply" or opname(nxt.op) not in ("add", "sum") or len(s.args) != 2:
            return False
        if nxt.value != s.name or s.name == nxt.name or nxt.base not in (None, nxt.name):
            return False
        if any(uses_name(t, s.name) for t in rest):
            return False
        if nxt.name not in self.env:
            self.bind(nxt.name, "f32", np.full(self.n, F32(identity_of(nxt.op))))
        self.bind(nxt.name, "f32", c_fma(self.f32(s.args[0]), self.f32(s.args[1]), self.f32(nxt.name)))
        return True

    def _fma_assign(self, s, nxt, rest) -> bool:
        if not (isinstance(s, Assign) and isinstance(nxt, Assign)):
            return False
        if opname(s.op) not in ("multiply", "mul") or opname(nxt.op) not in ("add", "sum"):
            return False
        if len(s.args) != 2 or len(nxt.args) != 2 or s.name not in nxt.args or s.name == nxt.name:
            return False
        if any(uses_name(t, s.name) for t in rest):
            return False
        other = nxt.args[0] if nxt.args[1] == s.name else nxt.args[1]
        self.bind(nxt.name, "f32", c_fma(self.f32(s.args[0]), self.f32(s.args[1]), self.f32(other)))
        return True

    def stmt(self, s) -> None:
        if isinstance(s, Load):
            dt = dtname(s.dtype) or self.dtypes.get(s.input)
            src = self.bufs[s.input]
            for k, name in enumerate(s.names):
                idx = np.broadcast_to(self.flat(s.input, self.idx_plus(s.index, k)), (self.n,))
                if self.mask is not None:
                    idx = np.where(self.mask, idx, 0)
                vals = src[idx]
                kind = "int" if dt in ("i32", "int", "int32", "s32", "u32") else "f32"
                self.bind(name, kind, vals.astype(np.int64) if kind == "int" else vals.astype(F32))
        elif isinstance(s, Write):
            dt = dtname(s.value_dtype) or self.dtypes.get(s.output)
            dst = self.bufs[s.output]
            for k, name in enumerate(s.values):
                idx = np.broadcast_to(self.flat(s.output, self.idx_plus(s.index, k)), (self.n,))
                vals = np.broadcast_to(store_cast(self.f32(name), dt), (self.n,))
                sel = slice(None) if self.mask is None else self.mask
                if s.atomic:
                    np.add.at(dst, idx[sel], vals[sel].astype(np.float64).astype(F32))
                else:
                    dst[idx[sel]] = vals[sel]
        elif isinstance(s, Let):
            dt = dtname(s.dtype)
            if dt in F32_NAMES or (dt is None and isinstance(s.value, Literal) and isinstance(s.value.value, float)):
                if isinstance(s.value, Literal):
                    self.bind(s.name, "f32", np.full(self.n, F32(float(s.value.value))))
                else:
                    self.bind(s.name, "f32", np.broadcast_to(self._tof(*self.expr(s.value)), (self.n,)))
            else:
                self.bind(s.name, "int", np.broadcast_to(self._toi(*self.expr(s.value)), (self.n,)))
        elif isinstance(s, Init):
            if dtname(s.dtype) in (None, *F32_NAMES):
                self.bind(s.name, "f32", np.full(self.n, F32(float(s.identity))))
            else:
                self.bind(s.name, "int", np.full(self.n, int(s.identity), np.int64))
        elif isinstance(s, Assign):
            op = opname(s.op)
            if dtname(s.dtype) in ("i32", "int", "int32", "s32", "u32"):
                a = [self._toi(*self._named(x)) for x in s.args]
                if op in ("add", "sum"):
                    v = a[0] + a[1]
                elif op in ("subtract", "sub"):
                    v = a[0] - a[1]
                elif op in ("multiply", "mul"):
                    v = a[0] * a[1]
                elif op in ("maximum", "max"):
                    v = np.maximum(a[0], a[1])
                elif op in ("minimum", "min"):
                    v = np.minimum(a[0], a[1])
                elif op in ("neg", "negative"):
                    v = -a[0]
                else:
                    v = np.abs(a[0])
                self.bind(s.name, "int", v)
            elif op == "where" and len(s.args) == 3:
                self.bind(s.name, "f32", np.where(self.pred(s.args[0]), self.f32(s.args[1]),
                                                  self.f32(s.args[2])).astype(F32))
            elif op in ("add", "sum", "subtract", "sub") and len(s.args) == 2 and (
                    self.product(s.args[0]) is not None or self.product(s.args[1]) is not None):
                sub = op in ("subtract", "sub")
                pa, pb = self.product(s.args[0]), self.product(s.args[1])
                if pa is not None and pb is not None:  # one fuses: the product defined last
                    if pa[2] > pb[2]:
                        pb = None
                    else:
                        pa = None
                if pa is not None:
                    c = self.f32(s.args[1])
                    v = c_fma(pa[0], pa[1], np.negative(c) if sub else c)
                else:
                    v = c_fma(np.negative(pb[0]) if sub else pb[0], pb[1], self.f32(s.args[0]))
                self.bind(s.name, "f32", np.broadcast_to(v, (self.n,)))
            else:
                fargs = [self.f32(a) for a in s.args]
                v = np.broadcast_to(f32_op(op, fargs), (self.n,))
                factors = None
                if op in ("multiply", "mul") and len(fargs) == 2:
                    factors = (fargs[0], fargs[1])
                elif op == "square":
                    factors = (fargs[0], fargs[0])
                elif op in ("log", "log_fast"):
                    factors = (lg2(fargs[0]), LN2)
                elif op == "silu":
                    e = ex2(np.multiply(np.negative(fargs[0]), LOG2E, dtype=F32))
                    factors = (fargs[0], np.divide(F32(1), np.add(F32(1), e, dtype=F32), dtype=F32))
                self.bind(s.name, "f32", v)
                if factors is not None:
                    self.order += 1
                    self.products[s.name] = (factors[0], factors[1], self.order)
        elif isinstance(s, Accum):
            if s.name not in self.env:
                self.bind(s.name, "f32", np.full(self.n, F32(identity_of(s.op))))
            left = self.f32(s.base) if s.base else self.f32(s.name)
            pv = self.product(s.value) if opname(s.op) in ("add", "sum") else None
            if pv is not None:
                self.bind(s.name, "f32", c_fma(pv[0], pv[1], left))
            else:
                self.bind(s.name, "f32", combine(opname(s.op), left, self.f32(s.value)))
        elif isinstance(s, Cond):
            p = np.broadcast_to(self._top(*self.expr(s.cond)), (self.n,))
            outer = self.mask
            self.mask = p if outer is None else (outer & p)
            self.run(s.body)
            if s.else_body:
                self.mask = ~p if outer is None else (outer & ~p)
                self.run(s.else_body)
            self.mask = outer
        elif isinstance(s, ZeroPrologue):
            # the kernel's own zero fill of `words` 32-bit words (compile.py:2890-2913)
            self.bufs[s.dst].view(np.uint32)[:int(s.words)] = 0
        elif isinstance(s, Loop):
            # sequential trips, every cell at once (the reference's per-thread loop order)
            for it in range(int(s.axis.extent.value)):
                self.env[s.axis.name] = ("int", np.int64(it))
                self.run(s.body)
        elif isinstance(s, Select):
            out = np.zeros(self.n, F32)
            taken = np.zeros(self.n, bool)
            for br in s.branches:
                p = np.broadcast_to(self._top(*self.expr(br.select)), (self.n,))
                out = np.where(~taken & p, self.f32(br.value), out)
                taken = taken | p
            self.bind(s.name, "f32", out)
        else:
            raise NotImplementedError(f"oracle: stmt {type(s).__name__}")

    def _named(self, x):
        if isinstance(x, str) and x in self.env:
            return self.env[x]
        return "f32", F32(float(x))


# ------------------------------------------------------------------ case driver


def load_case(case_dir: Path):
    case_dir = Path(case_dir)
    ir_path = next(case_dir.glob("*.ir.json"))
    raw = json.loads(ir_path.read_text())
    meta = json.loads((case_dir / "meta.json").read_text())
    graph = Graph.from_dict(raw)
    kop = next(n.op for n in graph.nodes.values() if isinstance(n.op, KernelOp))
    mk = meta["kernels"][0]
    shapes, dtypes = {}, {}
    for nd in raw["nodes"].values():
        for o in nd.get("outputs") or []:
            shapes[o["name"]] = tuple(o["shape"])
            dtypes[o["name"]] = o.get("dtype") or "f32"
    for a in mk.get("args") or []:
        shapes.setdefault(a["name"], tuple(a["shape"]))
        dtypes.setdefault(a["name"], a.get("dtype") or "f32")
    return kop, meta, mk, shapes, dtypes


def _axes(tile):
    return [(a.name, int(a.extent.value)) for a in tile.axes]


def _cells_for(axes, n_total):
    out = {}
    strides = row_major([e for _, e in axes])
    cell = np.arange(n_total, dtype=np.int64)
    for (name, e), st in zip(axes, strides):
        out[name] = (cell // st) % e
    return out


def evaluate(kop, shapes: dict, dtypes: dict, inputs: dict[str, np.ndarray],
             outputs: dict[str, tuple[int, ...]], launch: dict | None = None) -> dict[str, np.ndarray]:
    """Run ``kop`` on float32 ``inputs`` (bf16 inputs passed as their f32 values);
    returns float32 outputs (bf16/f16 outputs rounded as the store would).
    ``launch`` (meta ``grid``/``block``) sizes schedules whose threads do not
    all come from one Tile."""
    body = list(kop.body)
    nodes = list(ir_walk(body))
    if (any(isinstance(t, (CpAsyncCopy, CpAsyncCommit, CpAsyncWait, Pre, Carry)) for t in nodes)
            or not all(isinstance(t, Tile) for t in body)
            or (any(isinstance(t, Smem) for t in nodes)
                and not any(isinstance(t, (WarpShuffle, TreeHalve)) for t in nodes))
            or any(getattr(t, "aux_threads", 0) or getattr(t, "raster_group", None) for t in body)):
        return _eval_simt(kop, shapes, dtypes, inputs, outputs, launch)
    assert len(body) == 1 and isinstance(body[0], Tile), "oracle: one Tile per KernelOp"
    tile = body[0]
    stmts = list(tile.body)
    bufs = {k: np.ascontiguousarray(v, F32).reshape(-1) for k, v in inputs.items()}
    for name, shp in outputs.items():
        bufs[name] = np.zeros(int(np.prod(shp)) if shp else 1, F32)
    axes = _axes(tile)
    strided = [s for s in stmts if isinstance(s, StridedLoop)]
    loops = [s for s in stmts if isinstance(s, Loop)]
    if len(strided) > 1 or (strided and not any(isinstance(t, Accum) for t in ir_walk(strided[0].body))):
        _eval_phases(tile, stmts, axes, bufs, shapes, dtypes)
    elif strided:
        _eval_strided(tile, stmts, axes, strided[0], bufs, shapes, dtypes)
    elif loops and (len(loops) > 1 or any(isinstance(t, Loop) for t in ir_walk(loops[0].body))):
        # nested or several loops per cell (the naive attention IR): general sequential evaluation
        n = int(np.prod([e for _, e in axes])) if axes else 1
        m = Cells(n, bufs, shapes, dtypes)
        for k, v in _cells_for(axes, n).items():
            m.env[k] = ("int", v)
        m.run(stmts)
    elif loops and _is_matmul(loops[0]):
        _eval_matmul(tile, stmts, axes, loops[0], bufs, shapes, dtypes)
    elif loops:
        _eval_loop_reduce(tile, stmts, axes, loops[0], bufs, shapes, dtypes)
    else:
        n = int(np.prod([e for _, e in axes])) if axes else 1
        m = Cells(n, bufs, shapes, dtypes)
        for k, v in _cells_for(axes, n).items():
            m.env[k] = ("int", v)
        m.run(stmts)
    return {k: bufs[k].reshape(outputs[k]) if outputs[k] else bufs[k][:1] for k in outputs}


class Simt(Cells):
    """One thread block of a block-cooperative schedule, its threads as the
    vector lanes, run in lockstep (compile.py:1520-1629 thread model).

    Between barriers a race-free schedule gives the same values whatever the
    interleaving of its threads, so lockstep evaluation with the barriers as
    no-ops reproduces it.  Shared buffers live in ``bufs`` under their names
    for the duration of the block; ``cp.async`` copies complete at once."""

    def expr(self, e):
        if isinstance(e, Builtin):
            if e.name in self.env:
                return self.env[e.name]
            raise KeyError(f"oracle: thread builtin {e.name}")
        return super().expr(e)

    def stmt(self, s) -> None:
        if isinstance(s, (Smem, Sync, CpAsyncCommit, CpAsyncWait)):
            return
        if isinstance(s, StridedLoop):
            # per-thread start (compile.py:1866-1914): each lane runs its own trips
            start = np.broadcast_to(self._toi(*self.expr(s.start)), (self.n,)).astype(np.int64)
            step = np.broadcast_to(self._toi(*self.expr(s.step)), (self.n,)).astype(np.int64)
            end = (np.broadcast_to(self._toi(*self.expr(s.end)), (self.n,)) if s.end is not None
                   else np.full(self.n, int(s.axis.extent.value), np.int64))
            if s.seed:
                for t in s.body:
                    if isinstance(t, Accum) and t.name not in self.env:
                        self.bind(t.name, "f32", np.full(self.n, F32(identity_of(t.op))))
            outer = self.mask
            i = start.copy()
            while True:
                live = i < end
                if outer is not None:
                    live = live & outer
                if not live.any():
                    break
                self.mask = live
                self.env[s.axis.name] = ("int", i.copy())
                self.run(s.body)
                i = i + step
            self.mask = outer
            return
        if isinstance(s, Loop) and s.seed:
            for t in s.body:
                if isinstance(t, Accum) and t.name not in self.env:
                    self.bind(t.name, "f32", np.full(self.n, F32(identity_of(t.op))))
        if isinstance(s, WarpShuffle):
            lanes = np.arange(self.n, dtype=np.int64)
            step = int(s.length) // 2
            while step > 0:
                for st, sb in zip(s.state, s.state_b):
                    v = np.broadcast_to(self.f32(st), (self.n,))
                    self.env[sb] = ("f32", v[lanes ^ step].astype(F32))
                for asn in s.combine_states:
                    super().stmt(asn)
                step >>= 1
            return
        if isinstance(s, TreeHalve):
            tid = np.broadcast_to(self._toi(*self.expr(Var(s.tid_var))), (self.n,)).astype(np.int64)
            step = int(s.length) // 2

            def slot(extra):
                if s.inner is not None:
                    iv, scale = s.inner
                    return (tid + extra) * int(scale) + self._toi(*self.expr(Var(iv) if isinstance(iv, str) else iv))
                return tid + extra
            outer = self.mask
            while step > 0:
                take = tid < step
                if outer is not None:
                    take = take & outer
                self.mask = take
                for buf, st, sb in zip(s.bufs, s.state, s.state_b):
                    b = self.bufs[buf]
                    self.bind(st, "f32", b[np.where(take, slot(0), 0)].astype(F32))
                    self.bind(sb, "f32", b[np.where(take, slot(step), 0)].astype(F32))
                for asn in s.combine_states:
                    super().stmt(asn)
                for buf, st in zip(s.bufs, s.state):
                    b = self.bufs[buf]
                    vals = np.broadcast_to(self.f32(st), (self.n,))
                    b[slot(0)[take]] = vals[take]
                self.mask = outer
                step >>= 1
            for buf, st in zip(s.bufs, s.state):
                root = (self._toi(*self.expr(Var(s.inner[0]) if isinstance(s.inner[0], str) else s.inner[0]))
                        if s.inner is not None else 0)
                self.bind(st, "f32", np.broadcast_to(self.bufs[buf][root], (self.n,)).astype(F32))
            return
        if isinstance(s, Carry):
            v = np.broadcast_to(self.f32(s.value), (self.n,)).astype(F32)
            prod = self.products.get(s.value) if isinstance(s.value, str) else None
            self.carry_store[id(s)] = (v, prod)
            self.bind(s.name, "f32", v)
            return
        if isinstance(s, Pre):
            src, seed = self.carry_src.get(id(s), (None, 0.0))
            got = self.carry_store.get(src) if src is not None else None
            self.bind(s.name, "f32", got[0] if got is not None else np.full(self.n, F32(seed)))
            if got is not None and got[1] is not None:
                self.products[s.name] = got[1]    # a carried product stays foldable
            return
        if isinstance(s, CpAsyncCopy):
            # cp.async.ca|cg of nbytes (compile.py:2288-2319): f32 elements, contiguous
            dst, src = self.bufs[s.smem], self.bufs[s.src]
            didx = np.broadcast_to(self.flat(s.smem, s.smem_index), (self.n,)).astype(np.int64)
            if s.lane_index is not None:
                cols = int(self.shapes[s.smem][-1])
                didx = didx + (np.broadcast_to(self._toi(*self.expr(s.lane_index[0])), (self.n,)) * cols
                               + np.broadcast_to(self._toi(*self.expr(s.lane_index[1])), (self.n,)))
            sidx = np.broadcast_to(self.flat(s.src, s.src_index), (self.n,)).astype(np.int64)
            sel = np.ones(self.n, bool) if self.mask is None else self.mask
            for k in range(int(s.nbytes) // 4):
                dst[didx[sel] + k] = src[sidx[sel] + k]
            return
        super().stmt(s)


def _slot_of(index) -> str:
    """Carry slot of an index: a single literal index names its slot, else the wildcard (compile.py:2860-2866)."""
    if not index:
        return "0"
    if len(index) == 1 and isinstance(index[0], Literal) and isinstance(index[0].value, int):
        return str(index[0].value)
    return "_"


def _carry_sources(body) -> dict[int, tuple[int | None, float]]:
    """For every Pre, the Carry it reads and the seed it falls back to, as the
    reference resolves them while it emits code (compile.py:2860-2888): in
    program order, each loop body once, both branches of a Cond in turn."""
    vals: dict[tuple[str, str], int] = {}
    seeds: dict[str, float] = {}
    out: dict[int, tuple[int | None, float]] = {}

    def visit(stmts) -> None:
        for t in stmts:
            if isinstance(t, Carry):
                seeds[t.name] = float(t.seed)
                vals[(t.name, _slot_of(t.index))] = id(t)
            elif isinstance(t, Pre):
                key = (t.carrier, _slot_of(t.index))
                src = vals.get(key, vals.get((t.carrier, "_")))
                out[id(t)] = (src, seeds.get(t.carrier, 0.0))
            for child in (t.nested() if hasattr(t, "nested") else ()):
                visit(list(child))
    visit(list(body))
    return out


def _eval_simt(kop, shapes: dict, dtypes: dict, inputs: dict, outputs: dict, launch: dict | None = None):
    """Block-by-block lockstep evaluation of a block-cooperative KernelOp.
    Statements outside any Tile run in every thread of the meta launch."""
    launch = launch or {}
    bufs = {k: np.ascontiguousarray(v, F32).reshape(-1).copy() for k, v in inputs.items()}
    for name, shp in outputs.items():
        bufs[name] = np.zeros(int(np.prod(shp)) if shp else 1, F32)
    shapes = dict(shapes)
    smem = {}
    for t in ir_walk(list(kop.body)):
        if isinstance(t, Smem):
            smem[t.name] = tuple(int(x) for x in t.extents)
            shapes[t.name] = smem[t.name]
    carry_src = _carry_sources(list(kop.body))
    top = [t for t in kop.body if not isinstance(t, Smem)]
    tiles = [t for t in top if isinstance(t, Tile)]
    mblock = int(np.prod(launch.get("block") or [1])) if launch.get("block") else None
    mgrid = int(np.prod(launch.get("grid") or [1])) if launch.get("grid") else None

    def block_of(tile) -> int:
        return int(tile.block_threads or mblock or 128)

    if not tiles or any(not isinstance(t, Tile) for t in top):
        # one pass over the meta launch, every statement in order in every thread
        bt = mblock or (block_of(tiles[0]) if tiles else 1)
        nblocks = mgrid or max(1, -(-int(np.prod([a for _, a in _axes(tiles[0])])) // bt)) if tiles else (mgrid or 1)
        groups = [(bt, nblocks, top)]
    else:
        groups = []
        for tile in tiles:
            bt = block_of(tile)
            n_cells = int(np.prod([e for _, e in _axes(tile)])) if tile.axes else 1
            groups.append((bt, mgrid or max(1, -(-n_cells // bt)), [tile]))
    for bt, nblocks, stmts in groups:
        for b in range(nblocks):
            for name, shp in smem.items():
                bufs[name] = np.zeros(int(np.prod(shp)), F32)
            m = Simt(bt, bufs, shapes, dtypes)
            m.carry_src, m.carry_store = carry_src, {}
            tid = np.arange(bt, dtype=np.int64)
            gid = b * bt + tid
            m.env.update({"_tid": ("int", tid), "_gid": ("int", gid), "lane": ("int", tid & 31),
                          "warp": ("int", tid >> 5), "threadIdx.x": ("int", tid),
                          "blockIdx.x": ("int", np.full(bt, b, np.int64)), "blockDim.x": ("int", np.int64(bt))})
            for t in stmts:
                if not isinstance(t, Tile):
                    if isinstance(t, ZeroPrologue):
                        if b == 0:
                            bufs[t.dst].view(np.uint32)[:int(t.words)] = 0
                        continue
                    m.mask = None
                    m.stmt(t)
                    continue
                axes = _axes(t)
                n_cells = int(np.prod([e for _, e in axes])) if axes else 1
                for i, ((name, e), st) in enumerate(zip(axes, row_major([e for _, e in axes]))):
                    term = gid // st
                    m.env[name] = ("int", term if i == 0 else term % e)
                m.mask = (gid < n_cells) if (n_cells % bt or nblocks * bt != n_cells) else None
                m.run(list(t.body))
                m.mask = None
    return {k: bufs[k].reshape(outputs[k]) if outputs[k] else bufs[k][:1] for k in outputs}


def _is_matmul(loop) -> bool:
    loads = [s for s in loop.body if isinstance(s, Load)]
    return len(loads) == 2 and any(isinstance(s, Accum) for s in loop.body)


def _eval_matmul(tile, stmts, axes, loop, bufs, shapes, dtypes):
    (iname, M), (jname, N) = axes
    K = int(loop.axis.extent.value)
    kname = loop.axis.name
    la, lb = [s for s in loop.body if isinstance(s, Load)]
    ia = [ix.name for ix in la.index]
    ib = [ix.name for ix in lb.index]
    if ia[0] != iname:
        la, lb, ia, ib = lb, la, ib, ia
    A = bufs[la.input].reshape(M, K)
    b_nk = int(ib == [jname, kname])
    B = bufs[lb.input].reshape((N, K) if b_nk else (K, N))
    acc = np.empty((M, N), F32)
    A, B = np.ascontiguousarray(A), np.ascontiguousarray(B)
    lib().ora_gemm_seqfma_f32(_p(A), _p(B), _p(acc), M, N, K, b_nk)
    accum = next(s for s in loop.body if isinstance(s, Accum))
    i = stmts.index(loop)
    n = M * N
    m = Cells(n, bufs, shapes, dtypes)
    for k, v in _cells_for(axes, n).items():
        m.env[k] = ("int", v)
    m.env[accum.name] = ("f32", acc.reshape(-1))
    m.run([s for s in stmts[i + 1:]])


def _eval_loop_reduce(tile, stmts, axes, loop, bufs, shapes, dtypes):
    rows = int(np.prod([e for _, e in axes])) if axes else 1
    K = int(loop.axis.extent.value)
    kname = loop.axis.name
    # per-element values of the loop body, vectorised over rows x K
    n = rows * K
    m = Cells(n, bufs, shapes, dtypes)
    cells = _cells_for(axes + [(kname, K)], n)
    for k, v in cells.items():
        m.env[k] = ("int", v)
    body = list(loop.body)
    accs = [s for s in body if isinstance(s, Accum)]
    assert len(accs) == 1, "oracle: one accumulator in Loop reductions"
    acc = accs[0]
    m.count_uses(body)
    m.run([t for t in body if t is not acc])
    pv = m.product(acc.value) if opname(acc.op) in ("add", "sum") else None
    seed = identity_of(acc.op)
    for s in stmts[:stmts.index(loop)]:
        if isinstance(s, Init) and s.name == acc.name:
            seed = float(s.identity)
    out = np.empty(rows, F32)
    if pv is not None:
        xs = np.ascontiguousarray(np.broadcast_to(pv[0], (n,)), F32)
        ys = np.ascontiguousarray(np.broadcast_to(pv[1], (n,)), F32)
        lib().ora_loop_reduce_f32(_p(xs), _p(ys), rows, K, 4, F32(seed), _p(out))
    else:
        vals = np.ascontiguousarray(np.broadcast_to(m.f32(acc.value), (n,)), F32)
        op = {"add": 0, "sum": 0, "maximum": 1, "max": 1, "minimum": 2, "min": 2, "multiply": 3}[opname(acc.op)]
        lib().ora_loop_reduce_f32(_p(vals), None, rows, K, op, F32(seed), _p(out))
    pm = Cells(rows, bufs, shapes, dtypes)
    for k, v in _cells_for(axes, rows).items():
        pm.env[k] = ("int", v)
    pm.env[acc.name] = ("f32", out)
    pm.run(stmts[stmts.index(loop) + 1:])


def _eval_strided(tile, stmts, axes, loop, bufs, shapes, dtypes):
    co, bt = axes[-1]
    row_axes = axes[:-1]
    rows = int(np.prod([e for _, e in row_axes])) if row_axes else 1
    K = int(loop.axis.extent.value) if loop.end is None else int(loop.end.value)
    kname = loop.axis.name
    n = rows * K
    body = list(loop.body)
    accs = [s for s in body if isinstance(s, Accum)]
    results: dict[str, np.ndarray] = {}
    m = Cells(n, bufs, shapes, dtypes)
    for k, v in _cells_for(row_axes + [(kname, K)], n).items():
        m.env[k] = ("int", v)
    # element values; an Accum of a single-use product accumulates with fma
    # (the reference's multiply/Accum contraction, or ptxas fusing its mul/add pair)
    m.count_uses(body)
    m.run([t for t in body if not isinstance(t, Accum)])
    pending: list = []
    for acc in accs:
        pv = m.product(acc.value) if opname(acc.op) in ("add", "sum") else None
        if pv is not None:
            pending.append((acc, pv[0], pv[1]))
        else:
            pending.append((acc, np.broadcast_to(m.f32(acc.value), (n,)), None))
    opcode = {"add": 0, "sum": 0, "maximum": 1, "amax": 1, "max": 1, "minimum": 2, "amin": 2, "min": 2,
              "multiply": 3}
    for acc, x, y in pending:
        out = np.empty(rows, F32)
        xs = np.ascontiguousarray(np.broadcast_to(x, (n,)), F32)
        if y is not None:
            ys = np.ascontiguousarray(np.broadcast_to(y, (n,)), F32)
            lib().ora_strided_reduce_f32(_p(xs), _p(ys), rows, K, bt, 4, F32(0.0), _p(out))
        else:
            lib().ora_strided_reduce_f32(_p(xs), None, rows, K, bt, opcode[opname(acc.op)],
                                         F32(identity_of(acc.op)), _p(out))
        results[acc.name] = out
    # post statements: everything after the schedule, with co == 0 leader conds unwrapped
    i = stmts.index(loop)
    smem = {s.name for s in stmts if isinstance(s, Smem)}
    post = []
    for s in stmts[i + 1:]:
        if isinstance(s, (WarpShuffle, TreeHalve, Smem, Sync)):
            continue
        if isinstance(s, Cond):
            inner = list(s.body) + list(s.else_body)
            if inner and all(isinstance(t, Write) and t.output in smem for t in inner):
                continue
            c = s.cond
            if (isinstance(c, BinaryExpr) and c.op == "==" and isinstance(c.left, Var) and c.left.name == co):
                post.extend(s.body)
                continue
        post.append(s)
    pm = Cells(rows, bufs, shapes, dtypes)
    for k, v in _cells_for(row_axes, rows).items():
        pm.env[k] = ("int", v)
    for name, v in results.items():
        pm.env[name] = ("f32", v)
    pm.run(post)


def ir_walk(body):
    for t in body:
        yield t
        for child in t.nested():
            yield from ir_walk(child)


def _eval_phases(tile, stmts, axes, bufs, shapes, dtypes):
    """Block-per-row kernels with several strided passes over the row (fused
    reduction + pointwise: rmsnorm, softmax, l2norm).  Each reduction pass is
    the strided warp/tree schedule in the reference's exact order (as in
    ``_eval_strided``) and leaves its result in every thread; statements
    between passes are per-row scalars; a pass without Accum is pointwise over
    the row's elements and writes the output."""
    co, bt = axes[-1]
    row_axes = axes[:-1]
    rows = int(np.prod([e for _, e in row_axes])) if row_axes else 1
    smem = {t.name for t in stmts if isinstance(t, Smem)}
    pm = Cells(rows, bufs, shapes, dtypes)
    pm.count_uses(stmts)
    for k, v in _cells_for(row_axes, rows).items():
        pm.env[k] = ("int", v)
    opcode = {"add": 0, "sum": 0, "maximum": 1, "amax": 1, "max": 1, "minimum": 2, "amin": 2, "min": 2,
              "multiply": 3}
    row_stmts: list = []

    def flush():
        if row_stmts:
            pm.run(list(row_stmts))
            row_stmts.clear()

    for s in stmts:
        if isinstance(s, (WarpShuffle, TreeHalve, Smem, Sync)):
            continue
        if isinstance(s, Cond):
            inner = list(s.body) + list(s.else_body)
            if inner and all(isinstance(t, Write) and t.output in smem for t in inner):
                continue
            c = s.cond
            if isinstance(c, BinaryExpr) and c.op == "==" and isinstance(c.left, Var) and c.left.name == co:
                row_stmts.extend(s.body)
                continue
        if not isinstance(s, StridedLoop):
            row_stmts.append(s)
            continue
        flush()
        K = int(s.axis.extent.value) if s.end is None else int(s.end.value)
        n = rows * K
        m = Cells(n, bufs, shapes, dtypes)
        m.count_uses(stmts)
        for k, v in _cells_for(row_axes + [(s.axis.name, K)], n).items():
            m.env[k] = ("int", v)
        row_of = np.arange(n, dtype=np.int64) // K
        for name, (kind, v) in pm.env.items():
            if name not in m.env:
                v = np.asarray(v)
                m.env[name] = (kind, v[row_of] if v.ndim == 1 and v.shape[0] == rows else v)
        body = list(s.body)
        accs = [t for t in body if isinstance(t, Accum)]
        m.run([t for t in body if not isinstance(t, Accum)])
        for acc in accs:
            pv = m.product(acc.value) if opname(acc.op) in ("add", "sum") else None
            out = np.empty(rows, F32)
            if pv is not None:
                xs = np.ascontiguousarray(np.broadcast_to(pv[0], (n,)), F32)
                ys = np.ascontiguousarray(np.broadcast_to(pv[1], (n,)), F32)
                lib().ora_strided_reduce_f32(_p(xs), _p(ys), rows, K, bt, 4, F32(0.0), _p(out))
            else:
                xs = np.ascontiguousarray(np.broadcast_to(m.f32(acc.value), (n,)), F32)
                lib().ora_strided_reduce_f32(_p(xs), None, rows, K, bt, opcode[opname(acc.op)],
                                             F32(identity_of(acc.op)), _p(out))
            pm.bind(acc.name, "f32", out)
    flush()


def make_inputs(mk: dict, shapes: dict, dtypes: dict) -> dict[str, np.ndarray]:
    """Inputs from a meta kernel record: ``data`` literal, else ``init`` recipe
    with ``seed`` (default: standard normal, the reference tools' scheme,
    tools/make_proxy_set.py:62-67).  bf16 and f16 inputs are rounded to their type."""
    out = {}
    for a in mk.get("args") or []:
        if a.get("output"):
            continue
        shape = tuple(a.get("shape") or shapes.get(a["name"]) or (1,))
        if "data" in a:
            v = np.asarray(a["data"], F32).reshape(shape)
        else:
            rng = np.random.default_rng(int(a.get("seed", 0)))
            init = a.get("init") or {"kind": "normal", "mean": 0.0, "std": 1.0}
            if init["kind"] == "uniform":
                v = rng.uniform(init["low"], init["high"], size=shape).astype(F32)
            else:
                v = (rng.standard_normal(size=shape) * init.get("std", 1.0) + init.get("mean", 0.0)).astype(F32)
        if (a.get("dtype") or "f32") == "bf16":
            v = bf16_round(v).reshape(shape)
        elif (a.get("dtype") or "f32") == "f16":
            v = v.astype(np.float16).astype(F32)
        out[a["name"]] = v
    return out


def run_case(case_dir: Path, inputs: dict[str, np.ndarray] | None = None) -> tuple[dict, dict]:
    """Oracle outputs (and the inputs used) for a fixture directory."""
    kop, meta, mk, shapes, dtypes = load_case(case_dir)
    if inputs is None:
        inputs = make_inputs(mk, shapes, dtypes)
    outs = {a["name"]: tuple(a["shape"]) for a in mk["args"] if a.get("output")}
    res = evaluate(kop, shapes, dtypes, inputs, outs, {"grid": mk.get("grid"), "block": mk.get("block")})
    return res, inputs


def ulp_distance(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Distance in f32 units-in-the-last-place (0 for identical bits; NaNs
    compare equal to NaNs)."""
    a = np.ascontiguousarray(a, F32).reshape(-1)
    b = np.ascontiguousarray(b, F32).reshape(-1)
    ia = a.view(np.int32).astype(np.int64)
    ib = b.view(np.int32).astype(np.int64)
    ia = np.where(ia < 0, -(ia & 0x7FFFFFFF), ia)
    ib = np.where(ib < 0, -(ib & 0x7FFFFFFF), ib)
    d = np.abs(ia - ib)
    both_nan = np.isnan(a) & np.isnan(b)
    return np.where(both_nan, 0, d)


def within(got, ref, crit: dict) -> tuple[bool, str]:
    """Compare against an oracle criterion: {"ulp": n} (max f32 ulp distance)
    or {"rtol": r, "atol": a} (|got - ref| <= a + r |ref|, NaN == NaN)."""
    got = np.asarray(got, F32).reshape(-1)
    ref = np.asarray(ref, F32).reshape(-1)
    if "ulp" in crit:
        d = int(ulp_distance(got, ref).max()) if got.size else 0
        return d <= crit["ulp"], f"max {d} ulp (bound {crit['ulp']})"
    with np.errstate(invalid="ignore"):
        err = np.abs(got.astype(np.float64) - ref.astype(np.float64))
        bound = crit.get("atol", 0.0) + crit.get("rtol", 0.0) * np.abs(ref.astype(np.float64))
        bad = ~((err <= bound) | (np.isnan(got) & np.isnan(ref)))
    worst = float(np.nanmax(err - bound)) if got.size else 0.0
    return (not bad.any()), f"{int(bad.sum())} of {got.size} outside, worst excess {worst:.3g}"
