"""Per-cell CUDA C++ emission shared by the three kernel families.

The families decide *where* a cell's work runs (vector lanes, reduction
chunks, GEMM epilogue registers); this module decides *what* each IR
statement computes, and it must compute exactly what the reference compiler's
PTX computes for the same statement:

* the Assign op table and its rounding modes (compile.py:2068-2199): IEEE
  ``add/sub/mul`` with round-to-nearest (``__f*_rn``, which also keeps nvcc
  from contracting them), ``div.rn``, ``sqrt.rn``, ``rcp.rn``, and the
  approximate ``ex2.approx.ftz`` / ``lg2.approx.ftz`` / ``rsqrt.approx.ftz``
  instructions the reference builds exp/tanh/sigmoid/silu/log/pow from;
* the two FMA contraction peepholes: ``multiply`` followed by an ``Accum``
  add of the product (compile.py:1263-1283) and ``multiply`` followed by an
  ``add`` Assign that consumes it (compile.py:1285-1303), each only when the
  product is not read again later in the same statement list
  (compile.py:1415-1428);
* the contraction the reference's PTX gets from ptxas at load time: the
  reference emits plain ``mul.f32``/``add.f32``/``sub.f32`` (no rounding
  modifier, so the assembler may fuse them).  A plain product all of whose
  uses are plain add/sub (or Accum add) operands is fused into each of them,
  in any branch; when both operands of one add qualify, the later-defined
  product is the one fused (observed on B200 against the reference PTX, see
  :meth:`Emitter.plain_product`);
* f32 literal rounding (``f32_hex``, compile.py:205-207), accumulator seeds
  (``identity_of``, compile.py:327-338), ordered float compares
  (``setp.<cmp>.f32``) and truncating float->int casts (``cvt.rzi``);
* row-major flattening of multi-dimensional indices, a single index used
  as-is, and rank-mismatched indices summed (``flatten``,
  compile.py:2466-2493), with 64-bit arithmetic instead of the reference's
  s32.
"""

from __future__ import annotations

import math
import re
import struct

from . import ir
from .errors import UnsupportedIR

# ------------------------------------------------------------------ literals / types


def f32_bits(value: float) -> int:
    return struct.unpack(">I", struct.pack(">f", float(value)))[0]


def f32_lit(value: float) -> str:
    """Exact f32 constant (Python double rounded to nearest f32)."""
    return f"__uint_as_float(0x{f32_bits(value):08X}u)"


LOG2E_F32 = f32_lit(1.0 / math.log(2.0))
LN2_F32 = f32_lit(math.log(2.0))

CTYPE = {"f32": "float", "bf16": "__nv_bfloat16", "f16": "__half", "i32": "int", "u32": "unsigned",
         "f64": "double", "i64": "long long"}


def ctype(dt: str) -> str:
    try:
        return CTYPE[dt]
    except KeyError as exc:
        raise UnsupportedIR(f"unsupported element type {dt!r}") from exc


def load_to_kind(code: str, dt: str) -> tuple[str, str]:
    if dt == "f32":
        return "f32", code
    if dt == "bf16":
        return "f32", f"__bfloat162float({code})"
    if dt == "f16":
        return "f32", f"__half2float({code})"
    if dt in ("i32", "u32", "i64"):
        return "int", f"(long long)({code})"
    if dt == "f64":
        raise UnsupportedIR("f64 buffers are not lowered by the sm_100a families")
    raise UnsupportedIR(f"cannot load element type {dt!r}")


def store_from(kind: str, code: str, dt: str) -> str:
    if dt == "f32":
        return code if kind == "f32" else f"(float)({code})"
    if dt == "bf16":
        return f"__float2bfloat16_rn({code})" if kind == "f32" else f"__float2bfloat16_rn((float)({code}))"
    if dt == "f16":
        return f"__float2half_rn({code})" if kind == "f32" else f"__float2half_rn((float)({code}))"
    if dt in ("i32", "u32", "i64"):
        return f"({ctype(dt)})__float2int_rz({code})" if kind == "f32" else f"({ctype(dt)})({code})"
    raise UnsupportedIR(f"cannot store element type {dt!r}")


# ------------------------------------------------------------------ op table


IDENTITY = {"add": 0.0, "sum": 0.0, "multiply": 1.0, "prod": 1.0, "maximum": -1e30, "amax": -1e30,
            "max": -1e30, "minimum": 1e30, "min": 1e30}


def identity_of(op) -> float:
    """Accumulator seed of a combine op (compile.py:327-338): an explicit
    ``ElementwiseImpl.identity`` wins, else add 0, mul 1, max -1e30, min 1e30."""
    if not isinstance(op, str):
        ident = getattr(op, "identity", None)
        if ident is not None:
            return float(ident)
    return IDENTITY.get(ir.op_name(op), 0.0)


F32_BINARY = {"add": "__fadd_rn({a}, {b})", "sum": "__fadd_rn({a}, {b})",
              "subtract": "__fsub_rn({a}, {b})", "sub": "__fsub_rn({a}, {b})",
              "multiply": "__fmul_rn({a}, {b})", "mul": "__fmul_rn({a}, {b})",
              "divide": "__fdiv_rn({a}, {b})", "true_divide": "__fdiv_rn({a}, {b})",
              "div": "__fdiv_rn({a}, {b})",
              "maximum": "fmaxf({a}, {b})", "amax": "fmaxf({a}, {b})", "max": "fmaxf({a}, {b})",
              "minimum": "fminf({a}, {b})", "amin": "fminf({a}, {b})", "min": "fminf({a}, {b})"}
DIVIDE_OPS = ("divide", "true_divide", "div")
INT_BINARY = {"add": "({a} + {b})", "sum": "({a} + {b})", "subtract": "({a} - {b})",
              "sub": "({a} - {b})", "multiply": "({a} * {b})", "mul": "({a} * {b})",
              "maximum": "max({a}, {b})", "max": "max({a}, {b})", "minimum": "min({a}, {b})",
              "min": "min({a}, {b})"}
CMP = {"gt": ">", "greater": ">", "lt": "<", "less": "<", "ge": ">=", "greater_equal": ">=",
       "le": "<=", "less_equal": "<=", "eq": "==", "equal": "==", "ne": "!=", "not_equal": "!="}
INT_DTYPES = ("i32", "u32")


def f32_compare(op: str, a: str, b: str) -> str:
    """Ordered comparison, as ``setp.<cmp>.f32`` (false when either is NaN)."""
    if op == "!=":
        return f"(({a}) < ({b}) || ({a}) > ({b}))"
    return f"(({a}) {op} ({b}))"


def combine_code(op: str, a: str, b: str) -> str:
    """The Accum/combine instruction for ``op`` (F32_OPS, compile.py:140-155;
    unknown ops accumulate with add, compile.py:2209)."""
    return F32_BINARY.get(op, F32_BINARY["add"]).format(a=a, b=b)


# ------------------------------------------------------------------ names


_IDENT = re.compile(r"[^A-Za-z0-9_]")


def cname(name: str) -> str:
    return "v_" + _IDENT.sub("_", str(name))


# ------------------------------------------------------------------ index helpers


def row_major_strides(shape: tuple[int, ...]) -> list[int]:
    strides = [1] * len(shape)
    acc = 1
    for d in range(len(shape) - 1, -1, -1):
        strides[d] = acc
        acc *= int(shape[d])
    return strides


def lit_int(e) -> int | None:
    if isinstance(e, ir.Literal) and not isinstance(e.value, bool):
        if e.dtype in ("float", "f32"):
            return None
        if isinstance(e.value, int) or (isinstance(e.value, float) and e.value == int(e.value)):
            return int(e.value)
    return None


def uses_name(stmt, name: str) -> bool:
    """Does ``stmt`` (or anything nested in it) read IR name ``name``?
    Mirrors compile.py:1415-1428."""
    if isinstance(stmt, ir.Stmt) and name in stmt.reads():
        return True
    for child in stmt.nested() if isinstance(stmt, ir.Node) else ():
        for t in child:
            if uses_name(t, name):
                return True
    return False


PRODUCT_OPS = ("multiply", "mul", "square", "log", "log_fast", "silu")


def carry_slot(index) -> str:
    """The carry slot of a Carry/Pre index: a single literal index names its
    slot, anything else is the wildcard (compile.py:2860-2866)."""
    if not index:
        return "0"
    first = lit_int(index[0]) if len(index) == 1 else None
    if first is not None and all(lit_int(x) == 0 for x in index[1:]):
        return str(first)
    return "_"


def carry_aliases(body) -> dict[str, str]:
    """Names that are plain copies of another name through Carry / Pre: the
    reference emits both as ``mov.f32`` (compile.py:2868-2888), resolved in
    program order."""
    alias: dict[str, str] = {}
    carried: dict[tuple[str, str], str] = {}
    for t in ir.walk(body):
        if isinstance(t, ir.Carry) and isinstance(t.value, str):
            carried[(t.name, carry_slot(t.index))] = t.value
            alias[t.name] = t.value
        elif isinstance(t, ir.Pre):
            src = carried.get((t.carrier, carry_slot(t.index))) or carried.get((t.carrier, "_"))
            if src is not None:
                alias[t.name] = src
    return alias


def fusable_products(body) -> set[str]:
    """Names defined once by a plain-product Assign (``mul.f32`` in the
    reference's PTX) whose every read is an operand of a plain add/sub Assign
    or the value of an add Accum: the products the assembler folds into FMAs.
    Reads through Carry / Pre copies count as reads of the product (the
    assembler sees through the moves); the copies' names are returned too."""
    defs: dict[str, int] = {}
    for t in ir.walk(body):
        for name in _defined_names(t):
            defs[name] = defs.get(name, 0) + 1
    cands = {t.name for t in ir.walk(body)
             if isinstance(t, ir.Assign) and ir.op_name(t.op) in PRODUCT_OPS and defs.get(t.name) == 1}
    alias = carry_aliases(body)

    def root(n: str) -> str:
        for _ in range(len(alias) + 1):
            if n not in alias:
                break
            n = alias[n]
        return n

    bad: set[str] = set()
    for t in ir.walk(body):
        if not isinstance(t, ir.Stmt) or isinstance(t, ir.Carry):
            continue
        fusing = set()
        if isinstance(t, ir.Assign) and ir.op_name(t.op) in ("add", "sum", "subtract", "sub") and len(t.args) == 2:
            fusing = {a for a in t.args if isinstance(a, str)}
        elif isinstance(t, ir.Accum) and ir.op_name(t.op) in ("add", "sum") and t.base in (None, t.name):
            fusing = {t.value} if isinstance(t.value, str) else set()
        for n in _operand_reads(t):
            r = root(n)
            if r in cands and n not in fusing:
                bad.add(r)
    ok = cands - bad
    return ok | {n for n in alias if root(n) in ok}


def _defined_names(t) -> list[str]:
    if isinstance(t, ir.Load):
        return list(t.names)
    if isinstance(t, (ir.Assign, ir.Let, ir.Init, ir.Select)):
        return [t.name]
    return []


def _operand_reads(s) -> list[str]:
    """IR names a statement reads as instruction operands (one entry per read)."""
    out: list[str] = []
    if isinstance(s, ir.Assign):
        out += [a for a in s.args if isinstance(a, str)]
    elif isinstance(s, ir.Accum):
        out += [x for x in (s.value, s.base) if isinstance(x, str)]
    elif isinstance(s, ir.Write):
        out += [v for v in s.values if isinstance(v, str)]
        for ix in s.index:
            out += sorted(ix.var_names()) if isinstance(ix, ir.Expr) else []
    elif isinstance(s, ir.Select):
        for br in s.branches:
            if isinstance(br.value, str):
                out.append(br.value)
            if isinstance(br.select, ir.Expr):
                out += sorted(br.select.var_names())
    elif isinstance(s, (ir.Load, ir.Let, ir.Cond)):
        out += sorted(s.reads())
    return out


# ------------------------------------------------------------------ the emitter


class Emitter:
    """Translate straight-line IR statements (plus Cond/Select) into C++.

    ``env`` maps IR names to ``(kind, code)`` with kind in f32 / int / pred.
    ``load_hook(load, k)`` returns the C expression for the k-th name of a
    Load (the family decides whether that is a pre-fetched vector lane or a
    real memory access); ``write_hook(write, k, kind, code)`` returns the C
    statement for the k-th value of a Write.
    """

    def __init__(self, shapes: dict, dtypes: dict, ptrs: dict[str, str], load_hook=None,
                 write_hook=None, indent: str = "    "):
        self.shapes = shapes
        self.dtypes = dtypes
        self.ptrs = ptrs
        self.env: dict[str, tuple[str, str]] = {}
        self.lines: list[str] = []
        self.ind = indent
        self.load_hook = load_hook or self._default_load
        self.write_hook = write_hook or self._default_write
        self._hooks_given = (load_hook, write_hook)
        self.tmp = 0
        self.declared: dict[str, str] = {}
        # plain products (name -> (a, b) factor codes, definition order) and the
        # names whose every use is a plain add/sub operand
        self.products: dict[str, tuple[str, str, int]] = {}
        self.fusable: set[str] | None = None
        self.order = 0
        # C type of f32 values: "float", or "EmmyF2" when every value is a pair
        # of adjacent cells computed with packed f32x2 instructions
        self.ftype = "float"
        # divisor code -> (reciprocal code, fast-path flag code) for divisors shared by many cells
        self.row_divisors: dict[str, tuple[str, str]] = {}

    # -------------------------------------------------------------- small utils
    def emit(self, line: str) -> None:
        self.lines.append(self.ind + line)

    def fresh(self, stem: str = "t") -> str:
        self.tmp += 1
        return f"_{stem}{self.tmp}"

    def bind_const(self, name: str, kind: str, code: str) -> None:
        self.env[name] = (kind, code)

    def declare(self, name: str, kind: str) -> str:
        """A mutable C variable for IR name ``name`` (one per name and kind)."""
        key = f"{name}|{kind}"
        if key not in self.declared:
            var = cname(name) + ("" if kind == "f32" else "_" + kind)
            cty = {"f32": self.ftype, "int": "long long", "pred": "bool"}[kind]
            self.emit(f"{cty} {var};")
            self.declared[key] = var
        return self.declared[key]

    def assign(self, name: str, kind: str, code: str) -> str:
        self.products.pop(name, None)
        var = self.declare(name, kind)
        self.emit(f"{var} = {code};")
        self.env[name] = (kind, var)
        return var

    # -------------------------------------------------------------- values
    def as_f32(self, name) -> str:
        if isinstance(name, str) and name in self.env:
            kind, code = self.env[name]
            if kind == "f32":
                return code
            if kind == "int":
                return f"(float)({code})"
            return f"(({code}) ? 1.0f : 0.0f)"
        try:
            return f32_lit(float(name))
        except (TypeError, ValueError) as exc:
            raise UnsupportedIR(f"unknown f32 value {name!r}") from exc

    def as_int(self, name) -> str:
        if isinstance(name, str) and name in self.env:
            kind, code = self.env[name]
            if kind == "int":
                return code
            if kind == "f32":
                return f"(long long)__float2int_rz({code})"
            return f"(({code}) ? 1LL : 0LL)"
        return str(int(float(name)))

    def as_pred(self, name) -> str:
        if isinstance(name, str) and name in self.env and self.env[name][0] == "pred":
            return self.env[name][1]
        return f32_compare("!=", self.as_f32(name), "0.0f")

    # -------------------------------------------------------------- expressions
    def expr(self, e) -> tuple[str, str]:
        if isinstance(e, ir.Literal):
            v = e.value
            if isinstance(v, bool):
                return "int", "1LL" if v else "0LL"
            if e.dtype in ("int", "i32", "s32") or (isinstance(v, int) and e.dtype != "float"):
                return "int", f"{int(v)}LL"
            return "f32", f32_lit(float(v))
        if isinstance(e, ir.Var):
            if e.name in self.env:
                return self.env[e.name]
            raise UnsupportedIR(f"unbound var {e.name!r}")
        if isinstance(e, ir.Builtin):
            raise UnsupportedIR(f"thread builtin {e.name!r} depends on the reference schedule")
        if isinstance(e, ir.CastExpr):
            k, c = self.expr(e.expr)
            dt = ir.canon_dtype(e.dtype)
            if dt == "f32":
                return "f32", (c if k == "f32" else self._to_f32(k, c))
            return "int", (c if k == "int" else self._to_int(k, c))
        if isinstance(e, ir.TernaryExpr):
            p = self.pred_of(e.cond)
            tk, tc = self.expr(e.if_true)
            fk, fc = self.expr(e.if_false)
            if "f32" in (tk, fk):
                return "f32", f"({p} ? {self._to_f32(tk, tc)} : {self._to_f32(fk, fc)})"
            return "int", f"({p} ? {self._to_int(tk, tc)} : {self._to_int(fk, fc)})"
        if isinstance(e, ir.FuncCallExpr):
            args = []
            for a in e.args:
                k, c = self.expr(a)
                args.append(self._to_f32(k, c))
            return "f32", self.f32_op(e.name, args)
        if isinstance(e, ir.FlatIndex):
            return "int", self.flat_index(e.buffer, e.index)
        if isinstance(e, ir.BinaryExpr):
            return self.binary(e)
        raise UnsupportedIR(f"unsupported expr {type(e).__name__}")

    def _to_f32(self, kind: str, code: str) -> str:
        if kind == "f32":
            return code
        if kind == "int":
            return f"(float)({code})"
        return f"(({code}) ? 1.0f : 0.0f)"

    def _to_int(self, kind: str, code: str) -> str:
        if kind == "int":
            return code
        if kind == "f32":
            return f"(long long)__float2int_rz({code})"
        return f"(({code}) ? 1LL : 0LL)"

    def pred_of(self, e) -> str:
        k, c = self.expr(e)
        if k == "pred":
            return c
        if k == "f32":
            return f32_compare("!=", c, "0.0f")
        return f"(({c}) != 0)"

    def binary(self, e: ir.BinaryExpr) -> tuple[str, str]:
        op = e.op
        if op in ("&&", "||"):
            return "pred", f"({self.pred_of(e.left)} {op} {self.pred_of(e.right)})"
        lk, lc = self.expr(e.left)
        rk, rc = self.expr(e.right)
        if op in ("<", "<=", ">", ">=", "==", "!="):
            if "f32" in (lk, rk):
                return "pred", f32_compare(op, self._to_f32(lk, lc), self._to_f32(rk, rc))
            return "pred", f"(({self._to_int(lk, lc)}) {op} ({self._to_int(rk, rc)}))"
        if "f32" in (lk, rk):
            a, b = self._to_f32(lk, lc), self._to_f32(rk, rc)
            tbl = {"+": "__fadd_rn", "-": "__fsub_rn", "*": "__fmul_rn", "/": "__fdiv_rn",
                   "//": "__fdiv_rn"}
            if op not in tbl:
                raise UnsupportedIR(f"unsupported f32 binop {op!r}")
            return "f32", f"{tbl[op]}({a}, {b})"
        a, b = self._to_int(lk, lc), self._to_int(rk, rc)
        if op in ("+", "-", "*", "^", "&", "|"):
            return "int", f"(({a}) {op} ({b}))"
        if op in ("/", "//"):
            return "int", f"(({a}) / ({b}))"
        if op == "%":
            return "int", f"(({a}) % ({b}))"
        if op in ("<<", "shl"):
            return "int", f"(({a}) << ({b}))"
        if op in (">>", "shr"):
            return "int", f"(({a}) >> ({b}))"
        raise UnsupportedIR(f"unsupported binop {op!r}")

    def index_code(self, ix) -> str:
        k, c = self.expr(ix)
        return self._to_int(k, c)

    def flat_index(self, buf: str, indices) -> str:
        """Element offset of ``buf[indices]`` (compile.py:2466-2493)."""
        indices = tuple(indices)
        if not indices:
            return "0LL"
        shape = self.shapes.get(buf)
        if shape and len(indices) == 2 and len(shape) == 2:
            q, r = indices
            if (isinstance(q, ir.BinaryExpr) and isinstance(r, ir.BinaryExpr) and q.op in ("/", "//")
                    and r.op == "%" and lit_int(q.right) == int(shape[1]) == lit_int(r.right)
                    and q.left.pretty() == r.left.pretty()):
                return self.index_code(q.left)
        if len(indices) == 1:
            return self.index_code(indices[0])
        if not shape or len(shape) != len(indices):
            return "(" + " + ".join(f"({self.index_code(ix)})" for ix in indices) + ")"
        strides = row_major_strides(tuple(shape))
        terms = []
        for ix, st in zip(indices, strides):
            c = self.index_code(ix)
            terms.append(c if st == 1 else f"({c}) * {st}LL")
        return "(" + " + ".join(terms) + ")"

    def index_plus(self, indices, k: int) -> tuple:
        if k == 0:
            return tuple(indices)
        last = ir.BinaryExpr("+", indices[-1], ir.Literal(k, "int"))
        return tuple(indices[:-1]) + (last,)

    # -------------------------------------------------------------- memory hooks
    def _default_load(self, s: ir.Load, k: int) -> tuple[str, str]:
        dt = ir.canon_dtype(s.dtype or self.dtypes.get(s.input))
        idx = self.flat_index(s.input, self.index_plus(s.index, k))
        ptr = self.ptrs[s.input]
        return load_to_kind(f"{ptr}[{idx}]", dt)

    def _default_write(self, s: ir.Write, k: int, kind: str, code: str) -> str:
        dt = ir.canon_dtype(s.value_dtype or self.dtypes.get(s.output))
        idx = self.flat_index(s.output, self.index_plus(s.index, k))
        ptr = self.ptrs[s.output]
        if s.atomic:
            if dt != "f32":
                raise UnsupportedIR("atomic writes are f32 only (red.global.add.f32)")
            return f"atomicAdd(&{ptr}[{idx}], {self._to_f32(kind, code)});"
        return f"{ptr}[{idx}] = {store_from(kind, code, dt)};"

    # -------------------------------------------------------------- f32 op table
    def f32_op(self, op: str, args: list[str]) -> str:
        """One Assign op on already-f32 operands (compile.py:2087-2199)."""
        n = len(args)
        if op in DIVIDE_OPS and n == 2 and args[1] in self.row_divisors:
            r, ok = self.row_divisors[args[1]]
            return f"emmy_div_by({args[0]}, {args[1]}, {r}, {ok})"
        if op in F32_BINARY and n == 2:
            return F32_BINARY[op].format(a=args[0], b=args[1])
        if op in CMP and n == 2:
            return f"({f32_compare(CMP[op], args[0], args[1])} ? 1.0f : 0.0f)"
        if op == "exp2":
            return f"emmy_ex2_approx({args[0]})"
        if op in ("exp", "exp_fast"):
            return f"emmy_ex2_approx(__fmul_rn({args[0]}, {LOG2E_F32}))"
        if op == "sqrt":
            return f"__fsqrt_rn({args[0]})"
        if op == "rsqrt":
            return f"emmy_rsqrt_approx({args[0]})"
        if op in ("reciprocal", "recip"):
            return f"__frcp_rn({args[0]})"
        if op == "square" and n >= 1:
            return f"__fmul_rn({args[0]}, {args[0]})"
        if op in ("clamp", "clip") and n == 3:
            return f"fminf(fmaxf({args[0]}, {args[1]}), {args[2]})"
        if op == "relu":
            return f"fmaxf({args[0]}, 0.0f)"
        if op == "leaky_relu" and n >= 1:
            slope = args[1] if n > 1 else f32_lit(0.01)
            return f"emmy_leaky({args[0]}, {slope})"
        if op in ("neg", "negative"):
            return f"(-({args[0]}))"
        if op in ("abs", "absolute"):
            return f"fabsf({args[0]})"
        if op == "copy":
            return f"({args[0]})"
        if op in ("log", "log_fast"):
            return f"__fmul_rn(emmy_lg2_approx({args[0]}), {LN2_F32})"
        if op in ("log2", "lg2"):
            return f"emmy_lg2_approx({args[0]})"
        if op == "tanh":
            return f"emmy_tanh_ref({args[0]})"
        if op == "sigmoid":
            return f"emmy_sigmoid_ref({args[0]})"
        if op == "silu":
            return f"emmy_silu_ref({args[0]})"
        if op == "pow" and n == 2:
            return f"emmy_ex2_approx(__fmul_rn(emmy_lg2_approx({args[0]}), {args[1]}))"
        raise UnsupportedIR(f"unsupported assign op {op!r}")

    # -------------------------------------------------------------- statements
    def run(self, body) -> None:
        """Statement list with the reference's FMA lookahead (compile.py:1096-1131)."""
        if self.fusable is None:
            self.fusable = fusable_products(body)
        sl = list(ir.body_stmts(body))
        i = 0
        while i < len(sl):
            s = sl[i]
            nxt = sl[i + 1] if i + 1 < len(sl) else None
            rest = sl[i + 2:]
            if self.try_fma_accum(s, nxt, rest) or self.try_fma_assign(s, nxt, rest):
                i += 2
                continue
            self.stmt(s)
            i += 1

    def try_fma_accum(self, s, nxt, rest) -> bool:
        if not isinstance(s, ir.Assign) or not isinstance(nxt, ir.Accum):
            return False
        if ir.op_name(s.op) != "multiply" or ir.op_name(nxt.op) not in ("add", "sum") or len(s.args) != 2:
            return False
        if nxt.value != s.name or s.name == nxt.name or nxt.base not in (None, nxt.name):
            return False
        if any(uses_name(t, s.name) for t in rest):
            return False
        if nxt.name not in self.env:
            self.assign(nxt.name, "f32", f32_lit(identity_of(nxt.op)))
        acc = self.as_f32(nxt.name)
        a, b = self.as_f32(s.args[0]), self.as_f32(s.args[1])
        self.assign(nxt.name, "f32", f"__fmaf_rn({a}, {b}, {acc})")
        return True

    def try_fma_assign(self, s, nxt, rest) -> bool:
        if not isinstance(s, ir.Assign) or not isinstance(nxt, ir.Assign):
            return False
        if ir.op_name(s.op) not in ("multiply", "mul") or ir.op_name(nxt.op) not in ("add", "sum"):
            return False
        if len(s.args) != 2 or len(nxt.args) != 2:
            return False
        if s.name not in nxt.args or s.name == nxt.name:
            return False
        if any(uses_name(t, s.name) for t in rest):
            return False
        other = nxt.args[0] if nxt.args[1] == s.name else nxt.args[1]
        a, b, c = self.as_f32(s.args[0]), self.as_f32(s.args[1]), self.as_f32(other)
        self.assign(nxt.name, "f32", f"__fmaf_rn({a}, {b}, {c})")
        return True

    def stmt(self, s) -> None:
        if isinstance(s, ir.Load):
            for k, name in enumerate(s.names):
                kind, code = self.load_hook(s, k)
                self.assign(name, kind, code)
        elif isinstance(s, ir.Write):
            for k, name in enumerate(s.values):
                if isinstance(name, str) and name in self.env:
                    kind, code = self.env[name]
                else:
                    kind, code = "f32", self.as_f32(name)
                self.emit(self.write_hook(s, k, kind, code))
        elif isinstance(s, ir.Let):
            dt = ir.dtype_name(s.dtype)
            if dt in ir.F32_NAMES or (dt is None and isinstance(s.value, ir.Literal)
                                       and isinstance(s.value.value, float)):
                if isinstance(s.value, ir.Literal):
                    self.assign(s.name, "f32", f32_lit(float(s.value.value)))
                else:
                    k, c = self.expr(s.value)
                    self.assign(s.name, "f32", self._to_f32(k, c))
            else:
                k, c = self.expr(s.value)
                self.assign(s.name, "int", self._to_int(k, c))
        elif isinstance(s, ir.Init):
            if ir.canon_dtype(s.dtype) in ("f32",) or ir.dtype_name(s.dtype) is None:
                self.assign(s.name, "f32", f32_lit(float(s.identity)))
            else:
                self.assign(s.name, "int", f"{int(s.identity)}LL")
        elif isinstance(s, ir.Assign):
            self.emit_assign(s)
        elif isinstance(s, ir.Accum):
            if s.name not in self.env:
                self.assign(s.name, "f32", f32_lit(identity_of(s.op)))
            acc = self.as_f32(s.name)
            left = self.as_f32(s.base) if s.base else acc
            op = ir.op_name(s.op)
            prod = self.plain_product(s.value) if op in ("add", "sum") or op not in F32_BINARY else None
            if prod is not None:
                self.assign(s.name, "f32", f"__fmaf_rn({prod[0]}, {prod[1]}, {left})")
            else:
                self.assign(s.name, "f32", combine_code(op, left, self.as_f32(s.value)))
        elif isinstance(s, ir.Cond):
            p = self.pred_of(s.cond)
            # declare every name assigned inside either branch before the branch
            for t in list(ir.walk(s.body)) + list(ir.walk(s.else_body)):
                for nm, kind in self._defines(t):
                    self.declare(nm, kind)
            saved = dict(self.env)
            self.emit(f"if ({p}) {{")
            inner = self._child()
            inner.env = dict(saved)
            inner.run(s.body)
            self.lines.extend(inner.lines)
            self.env.update({k: v for k, v in inner.env.items() if k in self._vars_of(inner)})
            if s.else_body:
                self.emit("} else {")
                other = self._child()
                other.env = dict(saved)
                other.run(s.else_body)
                self.lines.extend(other.lines)
                self.env.update({k: v for k, v in other.env.items() if k in self._vars_of(other)})
            self.emit("}")
        elif isinstance(s, ir.Select):
            var = self.declare(s.name, "f32")
            taken = self.fresh("taken")
            self.emit(f"bool {taken} = false;")
            self.emit(f"{var} = 0.0f;")
            for br in s.branches:
                p = self.pred_of(br.select)
                val = self.as_f32(br.value)
                self.emit(f"if (!{taken} && {p}) {{ {var} = {val}; }}")
                self.emit(f"{taken} = {taken} || {p};")
            self.env[s.name] = ("f32", var)
        elif isinstance(s, (ir.Smem, ir.Sync)):
            raise UnsupportedIR(f"{type(s).__name__} is schedule state, not cell work")
        else:
            raise UnsupportedIR(f"unsupported stmt {type(s).__name__}")

    def _child(self) -> "Emitter":
        # custom hooks are shared; default ones are the child's own (its environment
        # holds the names a branch defines)
        c = Emitter(self.shapes, self.dtypes, self.ptrs, *self._hooks_given, self.ind + "    ")
        c.declared = self.declared
        c.tmp = self.tmp + 1000
        c.fusable = self.fusable
        c.products = self.products
        c.ftype = self.ftype
        return c

    @staticmethod
    def _vars_of(child: "Emitter") -> set[str]:
        return set(child.env)

    def _defines(self, s) -> list[tuple[str, str]]:
        if isinstance(s, ir.Load):
            dt = ir.canon_dtype(s.dtype or self.dtypes.get(s.input))
            kind = "int" if dt in INT_DTYPES else "f32"
            return [(n, kind) for n in s.names]
        if isinstance(s, ir.Assign):
            return [(s.name, self._assign_kind(s))]
        if isinstance(s, (ir.Accum, ir.Select)):
            return [(s.name, "f32")]
        if isinstance(s, ir.Init):
            return [(s.name, "f32" if ir.canon_dtype(s.dtype) == "f32" else "int")]
        if isinstance(s, ir.Let):
            dt = ir.dtype_name(s.dtype)
            f = dt in ir.F32_NAMES or (dt is None and isinstance(s.value, ir.Literal)
                                       and isinstance(s.value.value, float))
            return [(s.name, "f32" if f else "int")]
        return []

    @staticmethod
    def _assign_kind(s: ir.Assign) -> str:
        dt = ir.canon_dtype(s.dtype) if s.dtype is not None else "f32"
        return "int" if dt in INT_DTYPES else "f32"

    def emit_assign(self, s: ir.Assign) -> None:
        op = ir.op_name(s.op)
        args = list(s.args)
        if self._assign_kind(s) == "int":
            if op in INT_BINARY and len(args) == 2:
                a, b = self.as_int(args[0]), self.as_int(args[1])
                self.assign(s.name, "int", INT_BINARY[op].format(a=a, b=b))
                return
            if op in ("neg", "negative") and args:
                self.assign(s.name, "int", f"(-({self.as_int(args[0])}))")
                return
            if op in ("abs", "absolute") and args:
                self.assign(s.name, "int", f"llabs({self.as_int(args[0])})")
                return
        if op == "where" and len(args) == 3:
            p = self.as_pred(args[0])
            self.assign(s.name, "f32", f"({p} ? {self.as_f32(args[1])} : {self.as_f32(args[2])})")
            return
        if op in ("add", "sum", "subtract", "sub") and len(args) == 2:
            pa, pb = self.plain_product(args[0]), self.plain_product(args[1])
            if pa is not None and pb is not None:
                # the assembler fuses one: the product defined last
                if pa[2] > pb[2]:
                    pb = None
                else:
                    pa = None
            a, b = self.as_f32(args[0]), self.as_f32(args[1])
            sub = op in ("subtract", "sub")
            if pa is not None:
                self.assign(s.name, "f32", f"__fmaf_rn({pa[0]}, {pa[1]}, {'-(' + b + ')' if sub else b})")
                return
            if pb is not None:
                first = f"-({pb[0]})" if sub else pb[0]
                self.assign(s.name, "f32", f"__fmaf_rn({first}, {pb[1]}, {a})")
                return
        fargs = [self.as_f32(a) for a in args]
        factors = None
        if op in ("multiply", "mul") and len(fargs) == 2:
            factors = (fargs[0], fargs[1])
        elif op == "square" and fargs:
            factors = (fargs[0], fargs[0])
        elif op in ("log", "log_fast") and fargs:
            lg = self.fresh("lg2")
            self.emit(f"const {self.ftype} {lg} = emmy_lg2_approx({fargs[0]});")
            factors = (lg, LN2_F32)
        elif op == "silu" and fargs:
            sg = self.fresh("sig")
            self.emit(f"const {self.ftype} {sg} = emmy_sigmoid_ref({fargs[0]});")
            factors = (fargs[0], sg)
        if factors is not None:
            self.assign(s.name, "f32", f"__fmul_rn({factors[0]}, {factors[1]})")
            self.order += 1
            self.products[s.name] = (factors[0], factors[1], self.order)
            return
        self.assign(s.name, "f32", self.f32_op(op, fargs))

    def plain_product(self, name):
        """Factors of ``name`` if the reference computes it with a plain
        ``mul.f32``: the assembler fuses such a product into each plain
        add/sub that consumes it (the multiply is repeated per consumer when
        it has several), so the consumer is computed as one FMA."""
        if not isinstance(name, str) or name not in self.products:
            return None
        if self.fusable is not None and name not in self.fusable:
            return None
        if self.env.get(name, ("", ""))[1] != self.declared.get(f"{name}|f32"):
            return None
        return self.products[name]


DEVICE_PRELUDE = r"""
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

// x / y rounded to nearest (div.rn.f32, compile.py:2093) when many x share one
// divisor y whose reciprocal ry = RN(1 / y) (rcp.rn.f32) is computed once:
// Markstein's correction (P. Markstein, "Computation of elementary functions on
// the IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990):
// q0 = RN(x * ry) is within one ulp of x / y, the remainder r = x - q0 * y is
// exact in one fma, and RN(q0 + r * ry) is the correctly rounded quotient.  The
// fast path requires the operands, the quotient and the remainder to stay away
// from underflow and overflow (y_ok: 2^-64 <= |y| <= 2^64; |x| >= 2^-64;
// 2^-125 <= |q0| <= 2^126); everything else, zeros, infinities and NaNs
// included, takes __fdiv_rn itself.
static __device__ __forceinline__ bool emmy_div_ok(float y) {
    const float ay = fabsf(y);
    return ay >= 0x1p-64f && ay <= 0x1p+64f;
}
static __device__ __forceinline__ float emmy_div_by(float x, float y, float ry, bool y_ok) {
    const float q0 = __fmul_rn(x, ry);
    const float ax = fabsf(x), aq = fabsf(q0);
    if (!(y_ok && ax >= 0x1p-64f && aq >= 0x1p-125f && aq <= 0x1p+126f)) return __fdiv_rn(x, y);
    const float r = __fmaf_rn(-q0, y, x);
    return __fmaf_rn(r, ry, q0);
}

// Approximate-math instructions the reference compiler builds exp/tanh/
// sigmoid/silu/log/pow from (compile.py:2098-2195).  Issued as the same PTX
// instructions so results match bit for bit.
static __device__ __forceinline__ float emmy_ex2_approx(float x) {
    float y; asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x)); return y;
}
static __device__ __forceinline__ float emmy_lg2_approx(float x) {
    float y; asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x)); return y;
}
static __device__ __forceinline__ float emmy_rsqrt_approx(float x) {
    float y; asm("rsqrt.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x)); return y;
}
// tanh(x) = (2^(2x*log2e) - 1) / (2^(2x*log2e) + 1), compile.py:2142-2157.
// The reference rounds (x*2)*log2e; x*(2*log2e) (0x4038AA3B) is the same
// correctly rounded real product: doubling is exact, and where x*2 overflows
// both forms give +-inf.
static __device__ __forceinline__ float emmy_tanh_ref(float x) {
    float e = emmy_ex2_approx(__fmul_rn(x, __uint_as_float(0x4038AA3Bu)));
    return __fdiv_rn(__fsub_rn(e, 1.0f), __fadd_rn(e, 1.0f));
}
// sigmoid(x) = rcp(1 + 2^(-x*log2e)), compile.py:2158-2169.
static __device__ __forceinline__ float emmy_sigmoid_ref(float x) {
    float e = emmy_ex2_approx(__fmul_rn(-x, __uint_as_float(0x3FB8AA3Bu)));
    return __frcp_rn(__fadd_rn(1.0f, e));
}
// silu(x) = x * sigmoid(x), compile.py:2170-2183.
static __device__ __forceinline__ float emmy_silu_ref(float x) {
    return __fmul_rn(x, emmy_sigmoid_ref(x));
}
// leaky_relu: x > 0 ? x : x*slope, compile.py:2121-2129.
static __device__ __forceinline__ float emmy_leaky(float x, float slope) {
    float s = __fmul_rn(x, slope); return x > 0.0f ? x : s;
}

// Two adjacent cells in one value: add/sub/mul/fma go to the packed f32x2
// instructions (each lane rounded exactly as the scalar .rn instruction), the
// rest lane by lane.  a - b is computed as fma(b, -1, a): b*-1 is exact, so
// the single rounding of a - b is the same.  A float operand is broadcast.
struct EmmyF2 {
    float2 v;
    EmmyF2() = default;
    __device__ __forceinline__ EmmyF2(float s) : v(make_float2(s, s)) {}
    __device__ __forceinline__ EmmyF2(float2 p) : v(p) {}
};
#define EMMY_F2_LANES(f) make_float2(f(a.v.x), f(a.v.y))
static __device__ __forceinline__ EmmyF2 operator-(EmmyF2 a) { return make_float2(-a.v.x, -a.v.y); }
static __device__ __forceinline__ EmmyF2 __fadd_rn(EmmyF2 a, EmmyF2 b) { return __fadd2_rn(a.v, b.v); }
static __device__ __forceinline__ EmmyF2 __fmul_rn(EmmyF2 a, EmmyF2 b) { return __fmul2_rn(a.v, b.v); }
static __device__ __forceinline__ EmmyF2 __fmaf_rn(EmmyF2 a, EmmyF2 b, EmmyF2 c) {
    return __ffma2_rn(a.v, b.v, c.v);
}
static __device__ __forceinline__ EmmyF2 __fsub_rn(EmmyF2 a, EmmyF2 b) {
    return __ffma2_rn(b.v, make_float2(-1.0f, -1.0f), a.v);
}
static __device__ __forceinline__ EmmyF2 __fdiv_rn(EmmyF2 a, EmmyF2 b) {
    return make_float2(__fdiv_rn(a.v.x, b.v.x), __fdiv_rn(a.v.y, b.v.y));
}
static __device__ __forceinline__ EmmyF2 fmaxf(EmmyF2 a, EmmyF2 b) {
    return make_float2(fmaxf(a.v.x, b.v.x), fmaxf(a.v.y, b.v.y));
}
static __device__ __forceinline__ EmmyF2 fminf(EmmyF2 a, EmmyF2 b) {
    return make_float2(fminf(a.v.x, b.v.x), fminf(a.v.y, b.v.y));
}
static __device__ __forceinline__ EmmyF2 __frcp_rn(EmmyF2 a) { return EMMY_F2_LANES(__frcp_rn); }
static __device__ __forceinline__ EmmyF2 __fsqrt_rn(EmmyF2 a) { return EMMY_F2_LANES(__fsqrt_rn); }
static __device__ __forceinline__ EmmyF2 fabsf(EmmyF2 a) { return EMMY_F2_LANES(fabsf); }
static __device__ __forceinline__ EmmyF2 emmy_ex2_approx(EmmyF2 a) { return EMMY_F2_LANES(emmy_ex2_approx); }
static __device__ __forceinline__ EmmyF2 emmy_lg2_approx(EmmyF2 a) { return EMMY_F2_LANES(emmy_lg2_approx); }
static __device__ __forceinline__ EmmyF2 emmy_rsqrt_approx(EmmyF2 a) { return EMMY_F2_LANES(emmy_rsqrt_approx); }
static __device__ __forceinline__ EmmyF2 emmy_tanh_ref(EmmyF2 x) {
    const EmmyF2 e = emmy_ex2_approx(__fmul_rn(x, __uint_as_float(0x4038AA3Bu)));
    return __fdiv_rn(__fsub_rn(e, 1.0f), __fadd_rn(e, 1.0f));
}
static __device__ __forceinline__ EmmyF2 emmy_sigmoid_ref(EmmyF2 x) {
    const EmmyF2 e = emmy_ex2_approx(__fmul_rn(x, -__uint_as_float(0x3FB8AA3Bu)));
    return __frcp_rn(__fadd_rn(1.0f, e));
}
static __device__ __forceinline__ EmmyF2 emmy_silu_ref(EmmyF2 x) { return __fmul_rn(x, emmy_sigmoid_ref(x)); }
static __device__ __forceinline__ EmmyF2 emmy_leaky(EmmyF2 x, EmmyF2 slope) {
    return make_float2(emmy_leaky(x.v.x, slope.v.x), emmy_leaky(x.v.y, slope.v.y));
}
#undef EMMY_F2_LANES
"""

assert f32_bits(1.0 / math.log(2.0)) == 0x3FB8AA3B
assert f32_bits(2.0 / math.log(2.0)) == 0x4038AA3B
