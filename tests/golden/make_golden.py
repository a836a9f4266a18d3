#!/usr/bin/env python3
"""Generate the golden Kernel-IR fixtures and the reference compiler's PTX.

Run in a container that has the reference checkout (read-only) and the test
shim ``oracle/emmy_shim`` (it stands in for the absent ``emmy-ml`` package):

    python tests/golden/make_golden.py --reference /path/to/emmy-ptx-compiler

For every case this writes ``tests/golden/cases/<case>/``:

* ``<entry>.ir.json`` - an Emmy Graph whose KernelOp body is ``repr(body)``,
  exactly the layout the reference's fixture tools write
  (tools/make_proxy_set.py:42-55);
* ``meta.json`` - launch geometry, ``arg_order`` and per-argument input
  recipes, in the reference's meta schema (tools/make_proxy_set.py:75-86),
  plus an ``init`` recipe per input and a ``check`` block (tolerances);
* ``ref.ptx`` - what the unmodified reference ``compile.py`` prints for that
  IR (its ``compile_bundle``, compile.py:3168), when the reference can lower
  it.  bf16 GEMM IRs cannot be lowered by the reference (ptxas rejects its
  ``ld.global.nc.bf16`` form), so those cases carry a sibling ``ref_f32/``
  case: the same IR on fp32 copies of the operands, the oracle route for
  GEMM parity.

The IR shapes follow the reference's own generators: pointwise bodies
(make_proxy_set.py:89-213), the strided warp/tree reduction schedule
(make_proxy_set.py:215-336), the naive matmul (make_proxy_set.py:338-365) and
the extra op mixes of make_world_set.py:68-291.  They are rebuilt here with
our own code; nothing of the reference is copied into the repository except
the PTX its compiler prints for these inputs.

The GPU box has no reference checkout, so everything the tests need is
committed under ``tests/golden/cases``.
"""

from __future__ import annotations

import argparse
import importlib
import json
import math
import shutil
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
CASES = HERE / "cases"
BT = 128

sys.path.insert(0, str(REPO / "oracle" / "emmy_shim"))

import numpy as np  # noqa: E402
from emmy.compiler.dim import Dim  # noqa: E402
from emmy.compiler.ir.elementwise import ElementwiseImpl as EW  # noqa: E402
from emmy.compiler.ir.expr import BinaryExpr, Literal, Var  # noqa: E402
from emmy.compiler.ir.kernel.ir import (  # noqa: E402
    Axis, CpAsyncCommit, CpAsyncCopy, CpAsyncWait, DataType, Smem, Sync, Tile, TreeHalve, WarpShuffle,
)
from emmy.compiler.ir.expr import FlatIndex  # noqa: E402
from emmy.compiler.ir.stmt import (  # noqa: E402
    Accum, Assign, Carry, Cond, Init, Let, Load, Loop, Pre, StridedLoop, Write, ZeroPrologue,
)
from emmy.compiler.ir.stmt.leaves import Select, SelectBranch  # noqa: E402

F32 = DataType("f32", np.dtype("float32"), 4)
BF16 = DataType("bf16", None, 2)
F16 = DataType("f16", np.dtype("float16"), 2)


def _dt(dt: DataType) -> str:
    return dt.name


# ----------------------------------------------------------------- graph helpers


def _input(name: str, shape: list[int], dtype: str = "f32") -> dict:
    return {"op": "InputOp", "op_fields": {}, "inputs": [],
            "outputs": [{"name": name, "shape": shape, "dtype": dtype}]}


def _const(name: str, value: float) -> dict:
    return {"op": "ConstantOp",
            "op_fields": {"name": name, "value": value, "context_value": None, "load_ops": [],
                          "source_path": None, "source_parts": [], "source_shape": None,
                          "source_dtype": None, "source_graph": None},
            "inputs": [], "outputs": [{"name": name, "shape": [1], "dtype": "f32"}]}


def _kernel(entry: str, body, inputs: list[str], outputs: list[tuple[str, list[int], str]]) -> dict:
    return {"op": "KernelOp",
            "op_fields": {"body": [repr(body)], "name": entry, "zero_delegated": [], "serial": []},
            "inputs": inputs,
            "outputs": [{"name": n, "shape": s, "dtype": d} for n, s, d in outputs]}


def _launch(n: int, block: int = BT) -> tuple[list[int], list[int]]:
    return [max(1, math.ceil(n / block)), 1, 1], [block, 1, 1]


class Case:
    """One fixture directory."""

    def __init__(self, cid: str, entry: str, graph: dict, kernel: dict, *, family: str,
                 config: str | None = None, check: dict | None = None, ref: bool = True,
                 ref_case: "Case | None" = None, tags: tuple[str, ...] = ()):
        self.cid = cid
        self.entry = entry
        self.graph = graph
        self.kernel = kernel
        self.family = family
        self.config = config
        self.check = check or {}
        self.ref = ref
        self.ref_case = ref_case
        self.tags = tags

    def write(self, root: Path, compile_bundle) -> dict:
        d = root / self.cid
        if d.exists():
            shutil.rmtree(d)
        d.mkdir(parents=True)
        ir_path = d / f"{self.entry}.ir.json"
        ir_path.write_text(json.dumps(self.graph, indent=1) + "\n")
        meta = {"id": self.cid, "family": self.family, "config": self.config,
                "check": self.check, "tags": list(self.tags),
                "graph_inputs": self.graph["inputs"], "graph_outputs": self.graph["outputs"],
                "kernels": [self.kernel]}
        (d / "meta.json").write_text(json.dumps(meta, indent=1) + "\n")
        rec = {"id": self.cid, "entry": self.entry, "family": self.family, "config": self.config,
               "tags": list(self.tags), "ir": str(ir_path.relative_to(root)), "ref_ptx": None,
               "ref_case": None}
        if self.ref:
            bundle = compile_bundle(ir_path)
            (d / "ref.ptx").write_text(bundle["ptx"])
            rec["ref_ptx"] = str((d / "ref.ptx").relative_to(root))
        if self.ref_case is not None:
            sub = self.ref_case.write(d, compile_bundle)
            rec["ref_case"] = f"{self.cid}/{sub['id']}"
            rec["ref_ptx"] = f"{self.cid}/{sub['ref_ptx']}"
        return rec


def _arg(name: str, shape: list[int], dtype: str = "f32", *, init: dict | None = None,
         output: bool = False, seed: int | None = None) -> dict:
    a = {"name": name, "dtype": dtype, "shape": shape}
    if output:
        a["output"] = True
    else:
        a["seed"] = seed if seed is not None else 0
        a["init"] = init or {"kind": "normal", "mean": 0.0, "std": 1.0}
    return a


def _meta_kernel(node: str, entry: str, arg_order: list[str], grid, block, args: list[dict],
                 zero_outputs: list[str] | None = None) -> dict:
    return {"node": node, "entry": entry, "arg_order": arg_order, "grid": grid, "block": block,
            "smem_bytes": 0, "zero_outputs": zero_outputs or [], "args": args, "final": True}


# The reference builds exp/tanh/sigmoid/silu/log/rsqrt/pow from ex2/lg2/rsqrt.approx,
# whose exact bits are not published; the oracle uses correctly rounded libm
# instead, so for those IRs oracle == reference only up to the approximation
# error (amplified by cancellation, e.g. 1 + tanh(w) for w << 0).
APPROX_OPS = ("exp", "exp2", "tanh", "sigmoid", "silu", "log", "log2", "rsqrt", "pow")
APPROX_ORACLE = {"rtol": 4e-6, "atol": 2e-6}
UNIF = lambda lo, hi: {"kind": "uniform", "low": lo, "high": hi}  # noqa: E731
NORM = lambda std=1.0: {"kind": "normal", "mean": 0.0, "std": std}  # noqa: E731


# ------------------------------------------------------------------ config 1 / 2


def add_case(cid: str, n: int, *, block: int = 256, grid: int | None = None,
             config: str | None = None) -> Case:
    """c[i] = a[i] + b[i] (make_proxy_set.py:89-115 shape)."""
    entry = "k_add_pointwise"
    body = Tile(axes=(Axis("a0", Dim(n)),), body=(
        Load(names=("in0",), input="a", index=(Var("a0"),), dtype=F32),
        Load(names=("in1",), input="b", index=(Var("a0"),), dtype=F32),
        Assign("v0", EW("add"), ("in0", "in1"), F32),
        Write(output="c", index=(Var("a0"),), values=("v0",), value_dtype=F32),
    ))
    graph = {"inputs": ["a", "b"], "outputs": ["c"], "nodes": {
        "a": _input("a", [n]), "b": _input("b", [n]),
        "c": _kernel(entry, body, ["a", "b"], [("c", [n], "f32")])}}
    g = [grid if grid is not None else max(1, math.ceil(n / block)), 1, 1]
    kern = _meta_kernel("c", entry, ["a", "b", "c"], g, [block, 1, 1], [
        _arg("a", [n], init=UNIF(-1.0, 1.0), seed=0),
        _arg("b", [n], init=UNIF(-1.0, 1.0), seed=1),
        _arg("c", [n], output=True)])
    return Case(cid, entry, graph, kern, family="pointwise", config=config,
                check={"kind": "ulp", "ulp": 0})


def gelu_case(cid: str, rows: int, cols: int, *, config: str | None = None, dtype: DataType = F32) -> Case:
    """y = GELU_tanh(x*s + t) with per-column s, t.

    GELU-tanh has no IR op of its own, so the body is the Assign chain
    0.5*z*(1 + tanh(sqrt(2/pi)*(z + 0.044715*z^3))) with z = x*s + t; the
    reference contracts ``x*s``+``t`` and ``z3*c``+``z`` into fma.rn
    (compile.py:1285-1303) and lowers tanh through ex2.approx
    (compile.py:2142-2157).
    """
    entry = "k_gelu_tanh_affine"
    body = Tile(axes=(Axis("a0", Dim(rows)), Axis("a1", Dim(cols))), body=(
        Load(names=("xv",), input="x", index=(Var("a0"), Var("a1")), dtype=dtype),
        Load(names=("sv",), input="s", index=(Var("a1"),), dtype=dtype),
        Load(names=("tv",), input="t", index=(Var("a1"),), dtype=dtype),
        Assign("xs", EW("multiply"), ("xv", "sv"), F32),
        Assign("z", EW("add"), ("xs", "tv"), F32),
        Assign("z2", EW("multiply"), ("z", "z"), F32),
        Assign("z3", EW("multiply"), ("z2", "z"), F32),
        Let("c0", Literal(0.044715, "float"), F32),
        Assign("u0", EW("multiply"), ("z3", "c0"), F32),
        Assign("u", EW("add"), ("z", "u0"), F32),
        Let("c1", Literal(math.sqrt(2.0 / math.pi), "float"), F32),
        Assign("w", EW("multiply"), ("u", "c1"), F32),
        Assign("th", EW("tanh"), ("w",), F32),
        Let("one", Literal(1.0, "float"), F32),
        Assign("th1", EW("add"), ("th", "one"), F32),
        Let("half", Literal(0.5, "float"), F32),
        Assign("hz", EW("multiply"), ("z", "half"), F32),
        Assign("y0", EW("multiply"), ("hz", "th1"), F32),
        Write(output="y", index=(Var("a0"), Var("a1")), values=("y0",), value_dtype=dtype),
    ))
    graph = {"inputs": ["x", "s", "t"], "outputs": ["y"], "nodes": {
        "x": _input("x", [rows, cols], _dt(dtype)), "s": _input("s", [cols], _dt(dtype)),
        "t": _input("t", [cols], _dt(dtype)),
        "y": _kernel(entry, body, ["x", "s", "t"], [("y", [rows, cols], _dt(dtype))])}}
    grid, block = _launch(rows * cols)
    kern = _meta_kernel("y", entry, ["x", "s", "t", "y"], grid, block, [
        _arg("x", [rows, cols], _dt(dtype), init=NORM(), seed=0),
        _arg("s", [cols], _dt(dtype), init=UNIF(0.5, 1.5), seed=1),
        _arg("t", [cols], _dt(dtype), init=UNIF(-0.1, 0.1), seed=2),
        _arg("y", [rows, cols], _dt(dtype), output=True)])
    if dtype.name != "f32":
        # 16-bit loads and stores: the reference cannot lower them (ptxas rejects its
        # ld.global.nc.bf16 form), so parity is against the oracle, which rounds the same
        # f32 result to the output type (one output ulp apart at most)
        return Case(cid, entry, graph, kern, family="pointwise", config=config, ref=False,
                    check={"kind": "rtol", "rtol": 8e-3, "atol": 1e-3})
    return Case(cid, entry, graph, kern, family="pointwise", config=config,
                check={"kind": "ulp", "ulp": 1, "oracle": APPROX_ORACLE})


# ------------------------------------------------------------------ config 3 / 4


def _reduce_body(red_axis: Axis, start: str, index, accs: list[tuple[str, str]],
                 outs: list[tuple[str, tuple]], post=()) -> tuple:
    """The reference's strided warp/tree schedule (make_proxy_set.py:226-253),
    generalised to several accumulators sharing one pass over the input."""
    loads = (Load(names=("in0",), input="x", index=index, dtype=F32),)
    accums = tuple(Accum(a, "in0", EW(op), F32, axes=(red_axis.name,)) for a, op in accs)
    combine = tuple(Assign(a, EW(op), (a, f"{a}__o"), None) for a, op in accs)
    smems = tuple(Smem(f"{a}_smem", (BT // 32,), "float", 0) for a, _ in accs)
    lane_writes = tuple(Write(output=f"{a}_smem", index=(Var("warp"),), values=(a,), value_dtype=F32)
                        for a, _ in accs)
    final = tuple(Write(output=o, index=idx, values=(a,), value_dtype=F32)
                  for (a, _), (o, idx) in zip(accs, outs))
    return (
        # seed=True: accumulators start at their identity before the loop (compile.py:1868,
        # seed_accums 1769-1783); without it the reference seeds inside the loop body.
        StridedLoop(axis=red_axis, start=Var(start), step=Literal(BT, "int"), body=loads + accums,
                    seed=True),
        WarpShuffle(state=tuple(a for a, _ in accs), state_b=tuple(f"{a}__o" for a, _ in accs),
                    combine_states=combine, length=32, dtype=F32),
        *smems,
        Cond(BinaryExpr("==", Var("lane"), Literal(0, "int")), body=lane_writes),
        Sync(),
        TreeHalve(bufs=tuple(f"{a}_smem" for a, _ in accs), state=tuple(a for a, _ in accs),
                  state_b=tuple(f"{a}__o" for a, _ in accs), combine_states=combine,
                  length=BT // 32, tid_var="warp", dtype=F32),
        *post,
        Cond(BinaryExpr("==", Var(start), Literal(0, "int")), body=final),
    )


def _tree_phase(red_axis: Axis, start: str, body: tuple, acc: str, op: str) -> tuple:
    """One reduction phase of the strided warp/tree schedule whose result every
    thread of the block holds afterwards (TreeHalve re-reads the root slot,
    compile.py:2271-2277)."""
    comb = (Assign(acc, EW(op), (acc, f"{acc}__o"), None),)
    return (
        StridedLoop(axis=red_axis, start=Var(start), step=Literal(BT, "int"), body=body, seed=True),
        WarpShuffle(state=(acc,), state_b=(f"{acc}__o",), combine_states=comb, length=32, dtype=F32),
        Smem(f"{acc}_smem", (BT // 32,), "float", 0),
        Cond(BinaryExpr("==", Var("lane"), Literal(0, "int")),
             body=(Write(output=f"{acc}_smem", index=(Var("warp"),), values=(acc,), value_dtype=F32),)),
        Sync(),
        TreeHalve(bufs=(f"{acc}_smem",), state=(acc,), state_b=(f"{acc}__o",), combine_states=comb,
                  length=BT // 32, tid_var="warp", dtype=F32),
    )


def rownorm_case(cid: str, rows: int, cols: int, kind: str, *, config: str | None = None,
                 dtype: DataType = F32) -> Case:
    """Fused row reduction + pointwise epilogue, the rmsnorm / softmax / l2norm
    class (the reference's f01-f03): one block per row runs one or two
    reduction phases on the warp/tree schedule, then a strided pass that
    rereads the row and writes the normalised values."""
    ax = Axis("a1", Dim(cols))
    idx = (Var("a0"), Var("a1"))
    ld = lambda nm: Load(names=(nm,), input="x", index=idx, dtype=dtype)  # noqa: E731
    ins = ["x"]
    dn = _dt(dtype)
    if kind == "rmsnorm":
        entry = "k_rmsnorm"
        ins = ["x", "w"]
        phases = _tree_phase(ax, "a1_co", (ld("in0"), Assign("sq", EW("multiply"), ("in0", "in0"), F32),
                                           Accum("acc0", "sq", EW("add"), F32, axes=("a1",))), "acc0", "add")
        mid = (Let("inv_n", Literal(1.0 / cols, "float"), F32),
               Assign("ms", EW("multiply"), ("acc0", "inv_n"), F32),
               Let("eps", Literal(1e-6, "float"), F32),
               Assign("mse", EW("add"), ("ms", "eps"), F32),
               Assign("r", EW("rsqrt"), ("mse",), F32))
        tail = (ld("in1"), Load(names=("wv",), input="w", index=(Var("a1"),), dtype=dtype),
                Assign("xr", EW("multiply"), ("in1", "r"), F32),
                Assign("yv", EW("multiply"), ("xr", "wv"), F32))
    elif kind == "softmax":
        entry = "k_softmax"
        phases = _tree_phase(ax, "a1_co", (ld("in0"), Accum("acc0", "in0", EW("maximum"), F32, axes=("a1",))),
                             "acc0", "maximum")
        phases += _tree_phase(ax, "a1_co", (ld("in1"), Assign("d1", EW("subtract"), ("in1", "acc0"), F32),
                                            Assign("e1", EW("exp"), ("d1",), F32),
                                            Accum("acc1", "e1", EW("add"), F32, axes=("a1",))), "acc1", "add")
        mid = ()
        tail = (ld("in2"), Assign("d2", EW("subtract"), ("in2", "acc0"), F32),
                Assign("e2", EW("exp"), ("d2",), F32),
                Assign("yv", EW("divide"), ("e2", "acc1"), F32))
    elif kind == "l2norm":
        entry = "k_l2norm"
        phases = _tree_phase(ax, "a1_co", (ld("in0"), Assign("sq", EW("multiply"), ("in0", "in0"), F32),
                                           Accum("acc0", "sq", EW("add"), F32, axes=("a1",))), "acc0", "add")
        mid = (Let("eps", Literal(1e-12, "float"), F32),
               Assign("se", EW("add"), ("acc0", "eps"), F32),
               Assign("r", EW("rsqrt"), ("se",), F32))
        tail = (ld("in1"), Assign("yv", EW("multiply"), ("in1", "r"), F32))
    else:
        raise ValueError(kind)
    final = StridedLoop(axis=ax, start=Var("a1_co"), step=Literal(BT, "int"),
                        body=tail + (Write(output="y", index=idx, values=("yv",), value_dtype=dtype),))
    body = Tile(axes=(Axis("a0", Dim(rows)), Axis("a1_co", Dim(BT))), body=phases + mid + (final,),
                block_threads=BT)
    nodes = {"x": _input("x", [rows, cols], dn)}
    if "w" in ins:
        nodes["w"] = _input("w", [cols], dn)
    nodes["y"] = _kernel(entry, body, ins, [("y", [rows, cols], dn)])
    graph = {"inputs": ins, "outputs": ["y"], "nodes": nodes}
    args = [_arg("x", [rows, cols], dn, init=NORM(), seed=0)]
    if "w" in ins:
        args.append(_arg("w", [cols], dn, init=UNIF(0.5, 1.5), seed=1))
    args.append(_arg("y", [rows, cols], dn, output=True))
    kern = _meta_kernel("y", entry, ins + ["y"], [rows, 1, 1], [BT, 1, 1], args)
    # every kind uses an approximate instruction (rsqrt.approx, ex2.approx): the
    # oracle's libm stand-ins pin it within APPROX_ORACLE, not bit for bit
    check = {"kind": "rtol", "rtol": 1e-5, "atol": 1e-6, "oracle": APPROX_ORACLE}
    if dtype.name != "f32":
        # the reference cannot lower bf16 loads (ptxas rejects its ld.global.nc.bf16 form);
        # ours and the oracle round the same f32 result to bf16, up to one bf16 ulp apart
        check = {"kind": "rtol", "rtol": 8e-3, "atol": 1e-3}
    return Case(cid, entry, graph, kern, family="rownorm", config=config, check=check,
                ref=dtype.name == "f32")


def attention_case(cid: str, seq: int, dim: int, *, config: str | None = None, k_rows: bool = False) -> Case:
    """Naive attention, one thread per output cell (i, j) recomputing the
    scores three times: for the row max, for the softmax denominator, and
    for the weighted sum of V (the reference generator's a-class IR shape,
    tools/make_proxy_set.py:416-474).  q [seq, dim], kt = K^T [dim, seq],
    v [seq, dim], scale 1/sqrt(dim)."""
    entry = "k_attn_naive"
    scale = 1.0 / math.sqrt(dim)

    def scores(k: str, d: str, tag: str) -> tuple:
        return (
            Init(f"sc{tag}", 0.0, dtype=F32),
            Loop(axis=Axis(d, Dim(dim)), body=(
                Load(names=(f"q{tag}",), input="q", index=(Var("i"), Var(d)), dtype=F32),
                Load(names=(f"kt{tag}",), input="kt", index=((Var(k), Var(d)) if k_rows else (Var(d), Var(k))),
                     dtype=F32),
                Assign(f"p{tag}", EW("multiply"), (f"q{tag}", f"kt{tag}"), F32),
                Accum(f"sc{tag}", f"p{tag}", EW("add"), F32, axes=(d,)),
            )),
            Let(f"inv{tag}", Literal(scale, "float"), F32),
            Assign(f"sc{tag}", EW("multiply"), (f"sc{tag}", f"inv{tag}"), F32),
        )

    body = Tile(axes=(Axis("i", Dim(seq)), Axis("j", Dim(dim))), body=(
        Init("m", -1e30, dtype=F32),
        Loop(axis=Axis("k0", Dim(seq)), body=scores("k0", "d0", "0") + (
            Accum("m", "sc0", EW("maximum"), F32, axes=("k0",)),)),
        Init("den", 0.0, dtype=F32),
        Loop(axis=Axis("k1", Dim(seq)), body=scores("k1", "d1", "1") + (
            Assign("dl1", EW("subtract"), ("sc1", "m"), F32),
            Assign("ex1", EW("exp"), ("dl1",), F32),
            Accum("den", "ex1", EW("add"), F32, axes=("k1",)),)),
        Assign("invd", EW("reciprocal"), ("den",), F32),
        Init("acc", 0.0, dtype=F32),
        Loop(axis=Axis("k2", Dim(seq)), body=scores("k2", "d2", "2") + (
            Assign("dl2", EW("subtract"), ("sc2", "m"), F32),
            Assign("ex2", EW("exp"), ("dl2",), F32),
            Assign("wt", EW("multiply"), ("ex2", "invd"), F32),
            Load(names=("vv",), input="v", index=(Var("k2"), Var("j")), dtype=F32),
            Assign("wv", EW("multiply"), ("wt", "vv"), F32),
            Accum("acc", "wv", EW("add"), F32, axes=("k2",)),)),
        Write(output="attn", index=(Var("i"), Var("j")), values=("acc",), value_dtype=F32),
    ))
    ins = ["q", "kt", "v"]
    graph = {"inputs": ins, "outputs": ["attn"], "nodes": {
        "q": _input("q", [seq, dim]), "kt": _input("kt", [seq, dim] if k_rows else [dim, seq]),
        "v": _input("v", [seq, dim]),
        "attn": _kernel(entry, body, ins, [("attn", [seq, dim], "f32")])}}
    grid, block = _launch(seq * dim)
    kern = _meta_kernel("attn", entry, ins + ["attn"], grid, block, [
        _arg("q", [seq, dim], init=NORM(), seed=0),
        _arg("kt", [seq, dim] if k_rows else [dim, seq], init=NORM(), seed=1),
        _arg("v", [seq, dim], init=NORM(), seed=2), _arg("attn", [seq, dim], output=True)])
    return Case(cid, entry, graph, kern, family="attention", config=config,
                check={"kind": "rtol", "rtol": 1e-4, "atol": 1e-5, "oracle": APPROX_ORACLE})


def rowsummax_case(cid: str, rows: int, cols: int, *, config: str | None = None) -> Case:
    """row sum and row max of x[rows, cols] in one pass."""
    entry = "k_row_sum_max_reduce"
    body = Tile(axes=(Axis("a0", Dim(rows)), Axis("a1_co", Dim(BT))),
                body=_reduce_body(Axis("a1", Dim(cols)), "a1_co", (Var("a0"), Var("a1")),
                                  [("acc0", "add"), ("acc1", "maximum")],
                                  [("sum_1", (Var("a0"),)), ("max_1", (Var("a0"),))]),
                block_threads=BT)
    graph = {"inputs": ["x"], "outputs": ["sum_1", "max_1"], "nodes": {
        "x": _input("x", [rows, cols]),
        "sum_1": _kernel(entry, body, ["x"], [("sum_1", [rows], "f32"), ("max_1", [rows], "f32")])}}
    kern = _meta_kernel("sum_1", entry, ["x", "sum_1", "max_1"], [rows, 1, 1], [BT, 1, 1], [
        _arg("x", [rows, cols], init=NORM(), seed=0),
        _arg("sum_1", [rows], output=True), _arg("max_1", [rows], output=True)])
    return Case(cid, entry, graph, kern, family="reduction", config=config,
                check={"kind": "rtol", "rtol": 1e-5, "atol": 1e-5, "exact_outputs": ["max_1"]})


def fullsum_case(cid: str, n: int, *, config: str | None = None, ref: bool = True,
                 dist: dict | None = None) -> Case:
    """sum of x[n] (make_proxy_set.py:256-268 schedule, one block)."""
    entry = "k_sum_1_reduce"
    body = Tile(axes=(Axis("a0_co", Dim(BT)),),
                body=_reduce_body(Axis("a0", Dim(n)), "a0_co", (Var("a0"),), [("acc0", "add")],
                                  [("sum_1", ())]),
                block_threads=BT)
    graph = {"inputs": ["x"], "outputs": ["sum_1"], "nodes": {
        "x": _input("x", [n]), "sum_1": _kernel(entry, body, ["x"], [("sum_1", [], "f32")])}}
    kern = _meta_kernel("sum_1", entry, ["x", "sum_1"], [1, 1, 1], [BT, 1, 1], [
        _arg("x", [n], init=dist or UNIF(-1.0, 1.0), seed=0), _arg("sum_1", [1], output=True)])
    return Case(cid, entry, graph, kern, family="reduction", config=config, ref=ref,
                check={"kind": "rtol", "rtol": 1e-5, "atol": 1e-4})


def mean_case(cid: str, n: int) -> Case:
    """make_proxy_set.py:293-318: full mean = sum then multiply by 1/n."""
    entry = "k_mean_reduce"
    post = (Let("invn", Literal(1.0 / n, "float"), F32),
            Assign("acc0", EW("multiply"), ("acc0", "invn"), F32))
    body = Tile(axes=(Axis("a0_co", Dim(BT)),),
                body=_reduce_body(Axis("a0", Dim(n)), "a0_co", (Var("a0"),), [("acc0", "add")],
                                  [("mean", ())], post=post),
                block_threads=BT)
    graph = {"inputs": ["x"], "outputs": ["mean"], "nodes": {
        "x": _input("x", [n]), "mean": _kernel(entry, body, ["x"], [("mean", [], "f32")])}}
    kern = _meta_kernel("mean", entry, ["x", "mean"], [1, 1, 1], [BT, 1, 1], [
        _arg("x", [n], init=NORM(), seed=0), _arg("mean", [1], output=True)])
    return Case(cid, entry, graph, kern, family="reduction", check={"kind": "rtol", "rtol": 1e-5,
                                                                     "atol": 1e-6})


def fullmax_case(cid: str, n: int) -> Case:
    entry = "k_max_1_reduce"
    body = Tile(axes=(Axis("a0_co", Dim(BT)),),
                body=_reduce_body(Axis("a0", Dim(n)), "a0_co", (Var("a0"),), [("acc0", "maximum")],
                                  [("max_1", ())]),
                block_threads=BT)
    graph = {"inputs": ["x"], "outputs": ["max_1"], "nodes": {
        "x": _input("x", [n]), "max_1": _kernel(entry, body, ["x"], [("max_1", [], "f32")])}}
    kern = _meta_kernel("max_1", entry, ["x", "max_1"], [1, 1, 1], [BT, 1, 1], [
        _arg("x", [n], init=NORM(), seed=0), _arg("max_1", [1], output=True)])
    return Case(cid, entry, graph, kern, family="reduction", check={"kind": "exact"})


def rowsum_loop_case(cid: str, rows: int, cols: int) -> Case:
    """One thread per row, a plain ``Loop`` over the columns (no warp/tree stage)."""
    entry = "k_row_sumsq_loop"
    body = Tile(axes=(Axis("r", Dim(rows)),), body=(
        Init("acc", 0.0, dtype=F32),
        Loop(axis=Axis("c", Dim(cols)), body=(
            Load(names=("v",), input="x", index=(Var("r"), Var("c")), dtype=F32),
            Assign("sq", EW("multiply"), ("v", "v"), F32),
            Accum("acc", "sq", EW("add"), F32, axes=("c",)),
        )),
        Write(output="ss", index=(Var("r"),), values=("acc",), value_dtype=F32),
    ))
    graph = {"inputs": ["x"], "outputs": ["ss"], "nodes": {
        "x": _input("x", [rows, cols]), "ss": _kernel(entry, body, ["x"], [("ss", [rows], "f32")])}}
    grid, block = _launch(rows)
    kern = _meta_kernel("ss", entry, ["x", "ss"], grid, block, [
        _arg("x", [rows, cols], init=NORM(), seed=0), _arg("ss", [rows], output=True)])
    return Case(cid, entry, graph, kern, family="reduction", check={"kind": "rtol", "rtol": 1e-5,
                                                                     "atol": 1e-5})


def rowsum_loop_nonadjacent_case(cid: str, rows: int, cols: int) -> Case:
    """Loop reduction whose product and Accum are separated by a Let (no
    explicit fma.rn; the plain mul/add pair is left to the assembler)."""
    c = rowsum_loop_case(cid, rows, cols)
    entry = "k_row_sumsq_gap"
    body = Tile(axes=(Axis("r", Dim(rows)),), body=(
        Init("acc", 0.0, dtype=F32),
        Loop(axis=Axis("c", Dim(cols)), body=(
            Load(names=("v",), input="x", index=(Var("r"), Var("c")), dtype=F32),
            Assign("sq", EW("multiply"), ("v", "v"), F32),
            Let("z", Literal(0.0, "float"), F32),
            Accum("acc", "sq", EW("add"), F32, axes=("c",)),
        )),
        Write(output="ss", index=(Var("r"),), values=("acc",), value_dtype=F32),
    ))
    c.graph["nodes"]["ss"] = _kernel(entry, body, ["x"], [("ss", [rows], "f32")])
    c.entry = entry
    c.kernel["entry"] = entry
    return c


def atomic_sum_case(cid: str, n: int, *, zero_prologue: bool = False) -> Case:
    """make_world_set.py:247-266: every cell red.add's into sum_1[0].  With
    ``zero_prologue`` the kernel zeroes sum_1 itself (ZeroPrologue,
    compile.py:2890-2913) instead of the runner's zero_outputs."""
    entry = "k_atomic_sum"
    body = Tile(axes=(Axis("a0", Dim(n)),), body=(
        *((ZeroPrologue("sum_1", 1),) if zero_prologue else ()),
        Load(names=("in0",), input="x", index=(Var("a0"),), dtype=F32),
        Write(output="sum_1", index=(), values=("in0",), value_dtype=F32, atomic=True),
    ))
    graph = {"inputs": ["x"], "outputs": ["sum_1"], "nodes": {
        "x": _input("x", [n]), "sum_1": _kernel(entry, body, ["x"], [("sum_1", [], "f32")])}}
    grid, block = _launch(n)
    kern = _meta_kernel("sum_1", entry, ["x", "sum_1"], grid, block, [
        _arg("x", [n], init=NORM(), seed=0), _arg("sum_1", [1], output=True)],
        zero_outputs=[] if zero_prologue else ["sum_1"])
    return Case(cid, entry, graph, kern, family="reduction", check={"kind": "rtol", "rtol": 1e-5,
                                                                     "atol": 1e-4})


# ------------------------------------------------------------------ config 5


def gemm_case(cid: str, m: int, k: int, n: int, *, dtype: DataType = BF16, epilogue: bool = True,
              config: str | None = None, with_ref: bool = True, b_nk: bool = False) -> Case:
    """C = relu(A@B + bias), the naive matmul IR
    (make_proxy_set.py:338-365) plus a bias/ReLU epilogue.  bf16 operands and
    output, fp32 accumulate."""
    entry = "k_matmul_bias_relu" if epilogue else "k_matmul"
    out_dt = dtype
    tail: tuple = ()
    res = "acc0"
    if epilogue:
        tail = (Load(names=("bj",), input="bias", index=(Var("j"),), dtype=F32),
                Assign("v0", EW("add"), ("acc0", "bj"), F32),
                Assign("v1", EW("relu"), ("v0",), F32))
        res = "v1"
    body = Tile(axes=(Axis("i", Dim(m)), Axis("j", Dim(n))), body=(
        Init("acc0", 0.0, dtype=F32),
        Loop(axis=Axis("kk", Dim(k)), body=(
            Load(names=("a",), input="A", index=(Var("i"), Var("kk")), dtype=dtype),
            Load(names=("b",), input="B", index=((Var("j"), Var("kk")) if b_nk else (Var("kk"), Var("j"))),
                 dtype=dtype),
            Assign("p", EW("multiply"), ("a", "b"), F32),
            Accum("acc0", "p", EW("add"), F32, axes=("kk",)),
        )),
        *tail,
        Write(output="C", index=(Var("i"), Var("j")), values=(res,), value_dtype=out_dt),
    ))
    ins = ["A", "B"] + (["bias"] if epilogue else [])
    bshape = [n, k] if b_nk else [k, n]
    nodes = {"A": _input("A", [m, k], _dt(dtype)), "B": _input("B", bshape, _dt(dtype))}
    if epilogue:
        nodes["bias"] = _input("bias", [n], "f32")
    nodes["C"] = _kernel(entry, body, ins, [("C", [m, n], _dt(out_dt))])
    graph = {"inputs": ins, "outputs": ["C"], "nodes": nodes}
    grid, block = _launch(m * n)
    std = 0.02 if epilogue else 1.0
    args = [_arg("A", [m, k], _dt(dtype), init=NORM(std), seed=0),
            _arg("B", bshape, _dt(dtype), init=NORM(std), seed=1)]
    if epilogue:
        args.append(_arg("bias", [n], "f32", init=NORM(std), seed=2))
    args.append(_arg("C", [m, n], _dt(out_dt), output=True))
    kern = _meta_kernel("C", entry, ins + ["C"], grid, block, args)
    ref_case = None
    ref = True
    if dtype.name == "bf16":
        ref = False
        if with_ref:
            ref_case = gemm_case("ref_f32", m, k, n, dtype=F32, epilogue=epilogue, with_ref=False, b_nk=b_nk)
            ref_case.check = {"kind": "oracle_route",
                              "note": "fp32 copies of the bf16 operands; output rounded to bf16 RNE"}
    check = {"kind": "rtol", "rtol": 1e-2, "atol": 1e-2}
    if dtype.name == "f32":
        check = {"kind": "rtol", "rtol": 1e-5, "atol": 1e-5}
    return Case(cid, entry, graph, kern, family="gemm", config=config, check=check, ref=ref,
                ref_case=ref_case)


def cpasync_matmul_case(cid: str, m: int, k: int, n: int, *, wide: bool = False) -> Case:
    """A shared-memory matmul schedule of the kind Emmy emits with cp.async
    (lowered by compile.py:2288-2319, 1460-1465): one 16x16 output tile per
    256-thread block (Tile axes bi, bj, ty, tx), A and B staged tile by tile
    into shared memory by cp.async, then a sequential k loop over the staged
    tiles.  4-byte copies by every thread, or with ``wide`` 16-byte copies by
    the threads of the first four columns.  No reference generator writes this
    schedule; the IR is ours, its PTX is the reference compiler's."""
    ts = 16
    entry = "k_matmul_cpasync"
    lit = lambda v: Literal(v, "int")  # noqa: E731
    at = lambda blk, thr: BinaryExpr("+", BinaryExpr("*", Var(blk), lit(ts)), thr)  # noqa: E731
    row, col = at("bi", Var("ty")), at("bj", Var("tx"))
    if wide:
        tx4 = BinaryExpr("*", Var("tx"), lit(4))
        copies = (Cond(BinaryExpr("<", Var("tx"), lit(4)), body=(
            CpAsyncCopy("As", (Var("ty"), tx4), "A", (row, at("kt", tx4)), 16),
            CpAsyncCopy("Bs", (Var("ty"), tx4), "B", (at("kt", Var("ty")), at("bj", tx4)), 16),
        )),)
    else:
        copies = (CpAsyncCopy("As", (Var("ty"), Var("tx")), "A", (row, at("kt", Var("tx"))), 4),
                  CpAsyncCopy("Bs", (Var("ty"), Var("tx")), "B", (at("kt", Var("ty")), col), 4))
    body = Tile(axes=(Axis("bi", Dim(m // ts)), Axis("bj", Dim(n // ts)), Axis("ty", Dim(ts)),
                      Axis("tx", Dim(ts))), body=(
        Smem("As", (ts, ts), "float", 16),
        Smem("Bs", (ts, ts), "float", 16),
        Init("acc", 0.0, dtype=F32),
        Loop(axis=Axis("kt", Dim(k // ts)), body=(
            *copies,
            CpAsyncCommit(),
            CpAsyncWait(0),
            Sync(),
            Loop(axis=Axis("kk", Dim(ts)), body=(
                Load(names=("a",), input="As", index=(Var("ty"), Var("kk")), dtype=F32),
                Load(names=("b",), input="Bs", index=(Var("kk"), Var("tx")), dtype=F32),
                Assign("p", EW("multiply"), ("a", "b"), F32),
                Accum("acc", "p", EW("add"), F32, axes=("kk",)),
            )),
            Sync(),
        )),
        Write(output="C", index=(row, col), values=("acc",), value_dtype=F32),
    ), block_threads=ts * ts)
    graph = {"inputs": ["A", "B"], "outputs": ["C"], "nodes": {
        "A": _input("A", [m, k]), "B": _input("B", [k, n]),
        "C": _kernel(entry, body, ["A", "B"], [("C", [m, n], "f32")])}}
    grid = [(m // ts) * (n // ts), 1, 1]
    kern = _meta_kernel("C", entry, ["A", "B", "C"], grid, [ts * ts, 1, 1], [
        _arg("A", [m, k], init=NORM(), seed=0), _arg("B", [k, n], init=NORM(), seed=1),
        _arg("C", [m, n], output=True)])
    return Case(cid, entry, graph, kern, family="gemm", check={"kind": "ulp", "ulp": 0})


def raster_matmul_case(cid: str, m: int, k: int, n: int, group: int) -> Case:
    """The naive f32 matmul with a raster group on its Tile (compile.py:1563-1609):
    threads walk the (i, j) cells in groups of ``group`` rows."""
    entry = "k_matmul_raster"
    body = Tile(axes=(Axis("i", Dim(m)), Axis("j", Dim(n))), body=(
        Init("acc0", 0.0, dtype=F32),
        Loop(axis=Axis("kk", Dim(k)), body=(
            Load(names=("a",), input="A", index=(Var("i"), Var("kk")), dtype=F32),
            Load(names=("b",), input="B", index=(Var("kk"), Var("j")), dtype=F32),
            Assign("p", EW("multiply"), ("a", "b"), F32),
            Accum("acc0", "p", EW("add"), F32, axes=("kk",)),
        )),
        Write(output="C", index=(Var("i"), Var("j")), values=("acc0",), value_dtype=F32),
    ), raster_group=group, raster_axes=("i", "j"), raster_orient="m")
    graph = {"inputs": ["A", "B"], "outputs": ["C"], "nodes": {
        "A": _input("A", [m, k]), "B": _input("B", [k, n]),
        "C": _kernel(entry, body, ["A", "B"], [("C", [m, n], "f32")])}}
    grid, block = _launch(m * n)
    kern = _meta_kernel("C", entry, ["A", "B", "C"], grid, block, [
        _arg("A", [m, k], init=NORM(), seed=0), _arg("B", [k, n], init=NORM(), seed=1),
        _arg("C", [m, n], output=True)])
    return Case(cid, entry, graph, kern, family="gemm", check={"kind": "rtol", "rtol": 1e-5, "atol": 1e-5,
                                                                "exact_outputs": ["C"]})


def aux_threads_case(cid: str, n: int) -> Case:
    """A pointwise add whose Tile has 32 auxiliary threads per 128-thread
    block (compile.py:1528-1537).  The launch has 160 threads per block, as a
    32 x 5 block: the reference takes ``.reqntid`` from a multi-dimensional
    meta block, else from ``block_threads`` (compile.py:901-911).  The extra
    threads repeat cells of their block."""
    entry = "k_add_aux"
    body = Tile(axes=(Axis("a0", Dim(n)),), body=(
        Load(names=("u",), input="a", index=(Var("a0"),), dtype=F32),
        Load(names=("v",), input="b", index=(Var("a0"),), dtype=F32),
        Assign("w", EW("add"), ("u", "v"), F32),
        Write(output="c", index=(Var("a0"),), values=("w",), value_dtype=F32),
    ), block_threads=128, aux_threads=32)
    graph = {"inputs": ["a", "b"], "outputs": ["c"], "nodes": {
        "a": _input("a", [n]), "b": _input("b", [n]),
        "c": _kernel(entry, body, ["a", "b"], [("c", [n], "f32")])}}
    kern = _meta_kernel("c", entry, ["a", "b", "c"], [math.ceil(n / 128), 1, 1], [32, 5, 1], [
        _arg("a", [n], init=NORM(), seed=0), _arg("b", [n], init=NORM(), seed=1), _arg("c", [n], output=True)])
    return Case(cid, entry, graph, kern, family="schedule", check={"kind": "ulp", "ulp": 0})


def big_smem_case(cid: str, blocks: int, per_block: int) -> Case:
    """Each 256-thread block stages its slice of x in one shared buffer larger
    than 48 KiB, then writes the slice reversed.  The reference makes such a
    buffer ``.extern .shared`` sized by meta ``smem_bytes`` at launch
    (compile.py:827-836), which the harness passes (emmy_launch_ex)."""
    entry = "k_reverse_slices"
    t = 256
    lit = lambda v: Literal(v, "int")  # noqa: E731
    gidx = lambda e: BinaryExpr("+", BinaryExpr("*", Var("blk"), lit(per_block)), e)  # noqa: E731
    body = Tile(axes=(Axis("blk", Dim(blocks)), Axis("t", Dim(t))), body=(
        Smem("buf", (per_block,), "float", 16),
        StridedLoop(axis=Axis("e", Dim(per_block)), start=Var("t"), step=lit(t), body=(
            Load(names=("v",), input="x", index=(gidx(Var("e")),), dtype=F32),
            Write(output="buf", index=(Var("e"),), values=("v",), value_dtype=F32),
        )),
        Sync(),
        StridedLoop(axis=Axis("e2", Dim(per_block)), start=Var("t"), step=lit(t), body=(
            Load(names=("w",), input="buf",
                 index=(BinaryExpr("-", lit(per_block - 1), Var("e2")),), dtype=F32),
            Write(output="y", index=(gidx(Var("e2")),), values=("w",), value_dtype=F32),
        )),
    ), block_threads=t)
    n = blocks * per_block
    graph = {"inputs": ["x"], "outputs": ["y"], "nodes": {
        "x": _input("x", [n]), "y": _kernel(entry, body, ["x"], [("y", [n], "f32")])}}
    kern = _meta_kernel("y", entry, ["x", "y"], [blocks, 1, 1], [t, 1, 1], [
        _arg("x", [n], init=NORM(), seed=0), _arg("y", [n], output=True)])
    kern["smem_bytes"] = per_block * 4
    return Case(cid, entry, graph, kern, family="schedule", check={"kind": "exact"})


def cond_load_case(cid: str, n: int) -> Case:
    """A load inside a Cond whose index is a name the branch defines:
    y[i] = x[i] + x[i + n/2] for the first half, x[i]^2 for the rest."""
    entry = "k_cond_load"
    half = n // 2
    body = Tile(axes=(Axis("a0", Dim(n)),), body=(
        Load(names=("v",), input="x", index=(Var("a0"),), dtype=F32),
        Init("r", 0.0, dtype=F32),
        Cond(BinaryExpr("<", Var("a0"), Literal(half, "int")), body=(
            Let("k", BinaryExpr("+", Var("a0"), Literal(half, "int")), "i32"),
            Load(names=("w",), input="x", index=(Var("k"),), dtype=F32),
            Assign("r", EW("add"), ("v", "w"), F32),
        ), else_body=(
            Assign("r", EW("multiply"), ("v", "v"), F32),
        )),
        Write(output="y", index=(Var("a0"),), values=("r",), value_dtype=F32),
    ))
    graph = {"inputs": ["x"], "outputs": ["y"], "nodes": {
        "x": _input("x", [n]), "y": _kernel(entry, body, ["x"], [("y", [n], "f32")])}}
    grid, block = _launch(n)
    kern = _meta_kernel("y", entry, ["x", "y"], grid, block, [
        _arg("x", [n], init=NORM(), seed=0), _arg("y", [n], output=True)])
    return Case(cid, entry, graph, kern, family="pointwise", check={"kind": "ulp", "ulp": 0})


def smem_matmul_case(cid: str, m: int, k: int, n: int) -> Case:
    """The shared-memory matmul staged with plain copies: every thread of a
    16x16 block loads one element of the A tile and one of the B tile from
    global memory and stores it into shared memory, then a barrier, the k loop
    over the staged tiles, and a barrier before the next tile."""
    ts = 16
    entry = "k_matmul_smem"
    lit = lambda v: Literal(v, "int")  # noqa: E731
    at = lambda blk, thr: BinaryExpr("+", BinaryExpr("*", Var(blk), lit(ts)), thr)  # noqa: E731
    row, col = at("bi", Var("ty")), at("bj", Var("tx"))
    body = Tile(axes=(Axis("bi", Dim(m // ts)), Axis("bj", Dim(n // ts)), Axis("ty", Dim(ts)),
                      Axis("tx", Dim(ts))), body=(
        Smem("As", (ts, ts), "float", 16),
        Smem("Bs", (ts, ts), "float", 16),
        Init("acc", 0.0, dtype=F32),
        Loop(axis=Axis("kt", Dim(k // ts)), body=(
            Load(names=("ga",), input="A", index=(row, at("kt", Var("tx"))), dtype=F32),
            Write(output="As", index=(Var("ty"), Var("tx")), values=("ga",), value_dtype=F32),
            Load(names=("gb",), input="B", index=(at("kt", Var("ty")), col), dtype=F32),
            Write(output="Bs", index=(Var("ty"), Var("tx")), values=("gb",), value_dtype=F32),
            Sync(),
            Loop(axis=Axis("kk", Dim(ts)), body=(
                Load(names=("a",), input="As", index=(Var("ty"), Var("kk")), dtype=F32),
                Load(names=("b",), input="Bs", index=(Var("kk"), Var("tx")), dtype=F32),
                Assign("p", EW("multiply"), ("a", "b"), F32),
                Accum("acc", "p", EW("add"), F32, axes=("kk",)),
            )),
            Sync(),
        )),
        Write(output="C", index=(row, col), values=("acc",), value_dtype=F32),
    ), block_threads=ts * ts)
    graph = {"inputs": ["A", "B"], "outputs": ["C"], "nodes": {
        "A": _input("A", [m, k]), "B": _input("B", [k, n]),
        "C": _kernel(entry, body, ["A", "B"], [("C", [m, n], "f32")])}}
    kern = _meta_kernel("C", entry, ["A", "B", "C"], [(m // ts) * (n // ts), 1, 1], [ts * ts, 1, 1], [
        _arg("A", [m, k], init=NORM(), seed=0), _arg("B", [k, n], init=NORM(), seed=1),
        _arg("C", [m, n], output=True)])
    return Case(cid, entry, graph, kern, family="gemm", check={"kind": "ulp", "ulp": 0})


def pre_carry_case(cid: str, n: int) -> Case:
    """Values carried between statements by Carry and read back by Pre
    (compile.py:2860-2888): two slots of one carrier, and a carrier with no
    Carry that falls back to its seed (0)."""
    entry = "k_pre_carry"
    lit = lambda v: Literal(v, "int")  # noqa: E731
    body = Tile(axes=(Axis("a0", Dim(n)),), body=(
        Load(names=("v0",), input="x", index=(Var("a0"),), dtype=F32),
        Carry("c", "v0", (lit(0),), 0.0, F32),
        Assign("v1", EW("multiply"), ("v0", "v0"), F32),
        Carry("c", "v1", (lit(1),), 0.0, F32),
        Pre("p0", "c", (lit(0),)),
        Pre("p1", "c", (lit(1),)),
        Pre("p2", "d", (lit(0),)),
        Assign("s", EW("subtract"), ("p1", "p0"), F32),
        Assign("t", EW("add"), ("s", "p2"), F32),
        Write(output="y", index=(Var("a0"),), values=("t",), value_dtype=F32),
    ))
    graph = {"inputs": ["x"], "outputs": ["y"], "nodes": {
        "x": _input("x", [n]), "y": _kernel(entry, body, ["x"], [("y", [n], "f32")])}}
    grid, block = _launch(n)
    kern = _meta_kernel("y", entry, ["x", "y"], grid, block, [
        _arg("x", [n], init=NORM(), seed=0), _arg("y", [n], output=True)])
    return Case(cid, entry, graph, kern, family="schedule", check={"kind": "ulp", "ulp": 0})


def loose_statements_case(cid: str) -> Case:
    """Statements with no Tile around them, run by every thread of the launch:
    the kernel zeroes its output (ZeroPrologue), then every thread writes
    x[0] to out[0] through a FlatIndex Let, a Carry and a Pre (the node mix
    of the reference's tests/test_extra_isa.py:66-84)."""
    entry = "k_loose_nodes"
    lit = lambda v: Literal(v, "int")  # noqa: E731
    body = (
        ZeroPrologue("out", 32),
        Let("off", FlatIndex("x", (lit(0),)), "i32"),
        Load(names=("in0",), input="x", index=(Var("off"),), dtype=F32),
        Carry("st", "in0", (lit(0),), 0.0, F32),
        Pre("old", "st", (lit(0),)),
        Write(output="out", index=(lit(0),), values=("old",), value_dtype=F32),
    )
    graph = {"inputs": ["x"], "outputs": ["out"], "nodes": {
        "x": _input("x", [32]), "out": _kernel(entry, body, ["x"], [("out", [32], "f32")])}}
    kern = _meta_kernel("out", entry, ["x", "out"], [1, 1, 1], [32, 1, 1], [
        _arg("x", [32], init=NORM(), seed=0), _arg("out", [32], output=True)])
    return Case(cid, entry, graph, kern, family="schedule", check={"kind": "ulp", "ulp": 0})


# ------------------------------------------------------------ reference op catalog


def unary_case(cid: str, op: str, n: int, *, prep_abs: float | None = None, extra=()) -> Case:
    """make_proxy_set.py:118-142 / make_world_set.py:68-99 shapes."""
    entry = f"k_{op}_pointwise"
    pre: tuple = ()
    src = "in0"
    if prep_abs is not None:
        pre = (Assign("ab", EW("abs"), ("in0",), F32),
               Let("eps", Literal(prep_abs, "float"), F32),
               Assign("pz", EW("add"), ("ab", "eps"), F32))
        src = "pz"
    lets = tuple(Let(e, Literal(0.01, "float"), F32) for e in extra)
    body = Tile(axes=(Axis("a0", Dim(n)),), body=lets + (
        Load(names=("in0",), input="x", index=(Var("a0"),), dtype=F32),
        *pre,
        Assign("v0", EW(op), (src,) + tuple(extra), F32),
        Write(output="out", index=(Var("a0"),), values=("v0",), value_dtype=F32),
    ))
    graph = {"inputs": ["x"], "outputs": ["out"], "nodes": {
        "x": _input("x", [n]), "out": _kernel(entry, body, ["x"], [("out", [n], "f32")])}}
    grid, block = _launch(n)
    kern = _meta_kernel("out", entry, ["x", "out"], grid, block, [
        _arg("x", [n], init=NORM(), seed=0), _arg("out", [n], output=True)])
    approx = op in APPROX_OPS
    return Case(cid, entry, graph, kern, family="pointwise",
                check={"kind": "ulp", "ulp": 0, "oracle": APPROX_ORACLE if approx else {"ulp": 0}},
                tags=("catalog",))


def binary_case(cid: str, op: str, n: int) -> Case:
    entry = f"k_{op}_pointwise"
    body = Tile(axes=(Axis("a0", Dim(n)),), body=(
        Load(names=("in0",), input="x0", index=(Var("a0"),), dtype=F32),
        Load(names=("in1",), input="x1", index=(Var("a0"),), dtype=F32),
        Assign("v0", EW(op), ("in0", "in1"), F32),
        Write(output="out", index=(Var("a0"),), values=("v0",), value_dtype=F32),
    ))
    graph = {"inputs": ["x0", "x1"], "outputs": ["out"], "nodes": {
        "x0": _input("x0", [n]), "x1": _input("x1", [n]),
        "out": _kernel(entry, body, ["x0", "x1"], [("out", [n], "f32")])}}
    grid, block = _launch(n)
    kern = _meta_kernel("out", entry, ["x0", "x1", "out"], grid, block, [
        _arg("x0", [n], seed=0), _arg("x1", [n], seed=1), _arg("out", [n], output=True)])
    return Case(cid, entry, graph, kern, family="pointwise", check={"kind": "ulp", "ulp": 0},
                tags=("catalog",))


def chain_case(cid: str, n: int, which: str) -> Case:
    """Multi-statement pointwise mixes: relu_mul, scale_shift, leaky, clamp,
    where, select, cond_else, 2-D add, square_scale (make_proxy_set.py:145-213,
    367-390; make_world_set.py:164-245, 294-341)."""
    x = Load(names=("in0",), input="x", index=(Var("a0"),), dtype=F32)
    y = Load(names=("in1",), input="y", index=(Var("a0"),), dtype=F32)
    two_inputs = which in ("relu_mul", "where")
    if which == "relu_mul":
        stmts = (x, Assign("v0", EW("relu"), ("in0",), F32), y,
                 Assign("r", EW("multiply"), ("v0", "in1"), F32))
    elif which == "scale_shift":
        stmts = (x, Let("s", Literal(2.0, "float"), F32), Let("b", Literal(1.0, "float"), F32),
                 Assign("v0", EW("multiply"), ("in0", "s"), F32),
                 Assign("r", EW("add"), ("v0", "b"), F32))
    elif which == "leaky":
        stmts = (x, Let("z", Literal(0.0, "float"), F32), Let("s", Literal(0.01, "float"), F32),
                 Assign("p", EW("greater"), ("in0", "z"), F32),
                 Assign("sc", EW("multiply"), ("in0", "s"), F32),
                 Assign("r", EW("where"), ("p", "in0", "sc"), F32))
    elif which == "clamp":
        stmts = (x, Let("lo", Literal(-0.5, "float"), F32), Let("hi", Literal(0.5, "float"), F32),
                 Assign("t0", EW("maximum"), ("in0", "lo"), F32),
                 Assign("r", EW("minimum"), ("t0", "hi"), F32))
    elif which == "where":
        stmts = (x, y, Assign("p", EW("greater"), ("in0", "in1"), F32),
                 Assign("r", EW("where"), ("p", "in0", "in1"), F32))
    elif which == "select":
        stmts = (x, Let("z", Literal(0.0, "float"), F32),
                 Select("r", (SelectBranch("in0", BinaryExpr(">", Var("in0"), Var("z"))),
                              SelectBranch("z", Literal(1, "int")))))
    elif which == "cond_else":
        stmts = (x, Init("r", 0.0, dtype=F32),
                 Cond(BinaryExpr(">", Var("a0"), Literal(n // 2, "int")),
                      body=(Assign("r", EW("relu"), ("in0",), F32),),
                      else_body=(Assign("r", EW("negative"), ("in0",), F32),)))
    elif which == "square_scale":
        stmts = (x, Assign("v0", EW("square"), ("in0",), F32), Let("s", Literal(0.5, "float"), F32),
                 Assign("r", EW("multiply"), ("v0", "s"), F32))
    elif which == "silu_sigmoid":
        stmts = (x, Assign("sg", EW("sigmoid"), ("in0",), F32),
                 Assign("sl", EW("silu"), ("in0",), F32),
                 Assign("r", EW("add"), ("sg", "sl"), F32))
    elif which == "exp_log_sqrt":
        stmts = (x, Assign("ab", EW("abs"), ("in0",), F32), Let("e", Literal(1e-3, "float"), F32),
                 Assign("p", EW("add"), ("ab", "e"), F32), Assign("l", EW("log"), ("p",), F32),
                 Assign("q", EW("sqrt"), ("p",), F32), Assign("rq", EW("rsqrt"), ("p",), F32),
                 Assign("ex", EW("exp"), ("l",), F32), Assign("m", EW("multiply"), ("q", "rq"), F32),
                 Assign("d", EW("divide"), ("ex", "m"), F32), Assign("r", EW("add"), ("d", "l"), F32))
    elif which == "contract_square_add":
        # plain mul.f32 (square) whose only use is a plain add.f32
        stmts = (x, Assign("q", EW("square"), ("in0",), F32), Assign("r", EW("add"), ("q", "in0"), F32))
    elif which == "contract_nonadjacent":
        # multiply and add separated by a Let: no explicit fma.rn, plain mul/add pair
        stmts = (x, Let("c", Literal(1.5, "float"), F32), Assign("p", EW("multiply"), ("in0", "c"), F32),
                 Let("d", Literal(0.25, "float"), F32), Assign("r", EW("add"), ("p", "d"), F32))
    elif which == "contract_sub":
        stmts = (x, Let("c", Literal(1.5, "float"), F32), Assign("p", EW("multiply"), ("in0", "c"), F32),
                 Let("d", Literal(0.25, "float"), F32), Assign("r", EW("subtract"), ("d", "p"), F32))
    elif which == "contract_multiuse":
        # the product feeds two adds: not a single-use pair
        stmts = (x, Let("c", Literal(1.5, "float"), F32), Assign("p", EW("multiply"), ("in0", "c"), F32),
                 Assign("r1", EW("add"), ("p", "in0"), F32), Assign("r2", EW("subtract"), ("p", "c"), F32),
                 Assign("r", EW("multiply"), ("r1", "r2"), F32))
    elif which == "contract_two_products":
        # an add of two plain products: the assembler can fuse only one of them
        stmts = (x, Let("c", Literal(1.5, "float"), F32), Let("d", Literal(-0.75, "float"), F32),
                 Assign("p1", EW("multiply"), ("in0", "c"), F32), Assign("sq", EW("square"), ("in0",), F32),
                 Assign("p2", EW("multiply"), ("sq", "d"), F32), Assign("r", EW("add"), ("p1", "p2"), F32))
    elif which == "contract_two_products_swapped":
        # same products, the later-defined one is now the add's first operand
        stmts = (x, Let("c", Literal(1.5, "float"), F32), Let("d", Literal(-0.75, "float"), F32),
                 Assign("p1", EW("multiply"), ("in0", "c"), F32), Assign("sq", EW("square"), ("in0",), F32),
                 Assign("p2", EW("multiply"), ("sq", "d"), F32), Assign("r", EW("add"), ("p2", "p1"), F32))
    elif which == "contract_cond":
        # product defined before a Cond, consumed by adds inside both branches
        stmts = (x, Let("c", Literal(1.5, "float"), F32), Assign("p", EW("multiply"), ("in0", "c"), F32),
                 Init("r", 0.0, dtype=F32),
                 Cond(BinaryExpr(">", Var("a0"), Literal(n // 2, "int")),
                      body=(Assign("r", EW("add"), ("p", "in0"), F32),),
                      else_body=(Assign("r", EW("subtract"), ("p", "c"), F32),)))
    elif which == "contract_log_add":
        stmts = (x, Assign("ab", EW("abs"), ("in0",), F32), Let("e", Literal(1e-3, "float"), F32),
                 Assign("p", EW("add"), ("ab", "e"), F32), Assign("l", EW("log"), ("p",), F32),
                 Assign("r", EW("add"), ("l", "in0"), F32))
    else:
        raise ValueError(which)
    entry = f"k_{which}"
    body = Tile(axes=(Axis("a0", Dim(n)),), body=stmts + (
        Write(output="out", index=(Var("a0"),), values=("r",), value_dtype=F32),))
    ins = ["x", "y"] if two_inputs else ["x"]
    nodes = {i: _input(i, [n]) for i in ins}
    nodes["out"] = _kernel(entry, body, ins, [("out", [n], "f32")])
    graph = {"inputs": ins, "outputs": ["out"], "nodes": nodes}
    grid, block = _launch(n)
    args = [_arg(i, [n], seed=k) for k, i in enumerate(ins)] + [_arg("out", [n], output=True)]
    kern = _meta_kernel("out", entry, ins + ["out"], grid, block, args)
    approx = which in ("silu_sigmoid", "exp_log_sqrt", "contract_log_add")
    return Case(cid, entry, graph, kern, family="pointwise",
                check={"kind": "ulp", "ulp": 0, "oracle": APPROX_ORACLE if approx else {"ulp": 0}},
                tags=("catalog",))


def add2d_case(cid: str, h: int, w: int) -> Case:
    """make_proxy_set.py:186-212: 2-D add, one cell per (a0, a1)."""
    entry = "k_add2d_pointwise"
    body = Tile(axes=(Axis("a0", Dim(h)), Axis("a1", Dim(w))), body=(
        Load(names=("in0",), input="x0", index=(Var("a0"), Var("a1")), dtype=F32),
        Load(names=("in1",), input="x1", index=(Var("a0"), Var("a1")), dtype=F32),
        Load(names=("rb",), input="rowb", index=(Var("a0"),), dtype=F32),
        Assign("v0", EW("add"), ("in0", "in1"), F32),
        Assign("v1", EW("subtract"), ("v0", "rb"), F32),
        Write(output="out", index=(Var("a0"), Var("a1")), values=("v1",), value_dtype=F32),
    ))
    graph = {"inputs": ["x0", "x1", "rowb"], "outputs": ["out"], "nodes": {
        "x0": _input("x0", [h, w]), "x1": _input("x1", [h, w]), "rowb": _input("rowb", [h]),
        "out": _kernel(entry, body, ["x0", "x1", "rowb"], [("out", [h, w], "f32")])}}
    grid, block = _launch(h * w)
    kern = _meta_kernel("out", entry, ["x0", "x1", "rowb", "out"], grid, block, [
        _arg("x0", [h, w], seed=0), _arg("x1", [h, w], seed=1), _arg("rowb", [h], seed=2),
        _arg("out", [h, w], output=True)])
    return Case(cid, entry, graph, kern, family="pointwise", check={"kind": "ulp", "ulp": 0},
                tags=("catalog",))


def vec4_case(cid: str, n: int) -> Case:
    """make_world_set.py:102-131: the IR groups four consecutive cells."""
    entry = "k_add_v4"
    tiles = n // 4
    idx = lambda k: BinaryExpr("+", BinaryExpr("*", Var("a0"), Literal(4, "int")), Literal(k, "int"))  # noqa: E731
    stmts = []
    for k in range(4):
        stmts += [Load(names=(f"l{k}",), input="x0", index=(idx(k),), dtype=F32),
                  Load(names=(f"r{k}",), input="x1", index=(idx(k),), dtype=F32),
                  Assign(f"v{k}", EW("add"), (f"l{k}", f"r{k}"), F32)]
    body = Tile(axes=(Axis("a0", Dim(tiles)),), body=tuple(stmts) + (
        Write(output="out", index=(idx(0),), values=("v0", "v1", "v2", "v3"), value_dtype=F32),))
    graph = {"inputs": ["x0", "x1"], "outputs": ["out"], "nodes": {
        "x0": _input("x0", [n]), "x1": _input("x1", [n]),
        "out": _kernel(entry, body, ["x0", "x1"], [("out", [n], "f32")])}}
    grid, block = _launch(tiles)
    kern = _meta_kernel("out", entry, ["x0", "x1", "out"], grid, block, [
        _arg("x0", [n], seed=0), _arg("x1", [n], seed=1), _arg("out", [n], output=True)])
    return Case(cid, entry, graph, kern, family="pointwise", check={"kind": "ulp", "ulp": 0},
                tags=("catalog",))


def const_scale_case(cid: str, n: int) -> Case:
    """make_world_set.py:134-161: ConstantOp inputs read at index 0."""
    entry = "k_const_scale"
    body = Tile(axes=(Axis("a0", Dim(n)),), body=(
        Load(names=("c0",), input="mul_c", index=(Literal(0, "int"),), dtype=F32),
        Load(names=("c1",), input="add_c", index=(Literal(0, "int"),), dtype=F32),
        Load(names=("in0",), input="x", index=(Var("a0"),), dtype=F32),
        Assign("v0", EW("multiply"), ("in0", "c0"), F32),
        Assign("v1", EW("add"), ("v0", "c1"), F32),
        Write(output="out", index=(Var("a0"),), values=("v1",), value_dtype=F32),
    ))
    graph = {"inputs": ["x"], "outputs": ["out"], "nodes": {
        "mul_c": _const("mul_c", 3.0), "add_c": _const("add_c", -0.5), "x": _input("x", [n]),
        "out": _kernel(entry, body, ["mul_c", "add_c", "x"], [("out", [n], "f32")])}}
    grid, block = _launch(n)
    kern = _meta_kernel("out", entry, ["mul_c", "add_c", "x", "out"], grid, block, [
        {"name": "mul_c", "dtype": "f32", "shape": [1], "data": [3.0]},
        {"name": "add_c", "dtype": "f32", "shape": [1], "data": [-0.5]},
        _arg("x", [n], seed=0), _arg("out", [n], output=True)])
    return Case(cid, entry, graph, kern, family="pointwise", check={"kind": "ulp", "ulp": 0},
                tags=("catalog",))


def launch3d_case(cid: str, n: int = 64) -> Case:
    """make_world_set.py:269-291: a 3-D block launch of a 1-D Tile."""
    c = binary_case(cid, "add", n)
    c.entry = "k_add_3d"
    c.kernel["entry"] = "k_add_3d"
    body_node = c.graph["nodes"]["out"]
    body_node["op_fields"]["name"] = "k_add_3d"
    c.kernel["grid"] = [1, 1, 1]
    c.kernel["block"] = [8, 4, 2]
    return c


# ------------------------------------------------------------------ registry


def all_cases() -> list[Case]:
    cases: list[Case] = []
    # config 1
    cases.append(add_case("c1_add_64", 64, block=256, grid=1, config="c1"))
    cases.append(add_case("c1_add_1000", 1000))
    # config 2
    cases.append(gelu_case("c2_gelu_full", 16384, 16384, config="c2"))
    cases.append(gelu_case("c2_gelu_prof_4096x16384", 4096, 16384))  # > L2, for profiler captures
    cases.append(gelu_case("c2_gelu_256x4096", 256, 4096))
    cases.append(gelu_case("c2_gelu_64x1000", 64, 1000))
    cases.append(gelu_case("c2_gelu_3x7", 3, 7))
    cases.append(gelu_case("c2_gelu_1x1", 1, 1))
    cases.append(gelu_case("p_gelu_bf16_64x1000", 64, 1000, dtype=BF16))
    cases.append(gelu_case("p_gelu_f16_7x36", 7, 36, dtype=F16))
    # config 3
    cases.append(rowsummax_case("c3_rowsummax_full", 8192, 65536, config="c3"))
    cases.append(rowsummax_case("c3_rowsummax_64x5000", 64, 5000))
    cases.append(rowsummax_case("c3_rowsummax_16x65536", 16, 65536))
    cases.append(rowsummax_case("c3_rowsummax_300x200", 300, 200))
    cases.append(rowsummax_case("c3_rowsummax_5x64", 5, 64))
    # config 4 (the reference indexes in s32, so it cannot lower n = 2^31 as one launch;
    # its oracle route is 2^28-element chunks)
    cases.append(fullsum_case("c4_sum_full", 1 << 31, config="c4", ref=False))
    cases.append(fullsum_case("c4_sum_chunk_2p28", 1 << 28))
    cases.append(fullsum_case("c4_sum_1048579", (1 << 20) + 3))
    cases.append(fullsum_case("c4_sum_1000", 1000))
    cases.append(fullsum_case("c4_sum_1", 1))
    cases.append(mean_case("r_mean_777", 777))
    cases.append(fullmax_case("r_max_1024", 1024))
    cases.append(rowsum_loop_case("r_rowsumsq_loop_33x250", 33, 250))
    cases.append(rowsum_loop_nonadjacent_case("r_rowsumsq_gap_17x300", 17, 300))
    cases.append(atomic_sum_case("r_atomic_sum_512", 512))
    # one block: the reference's in-kernel zero fill races with other blocks' adds otherwise
    cases.append(atomic_sum_case("r_atomic_zp_sum_128", 128, zero_prologue=True))
    # config 5
    cases.append(gemm_case("c5_gemm_full", 16384, 8192, 16384, config="c5"))
    cases.append(gemm_case("c5_gemm_prof_8192x8192x8192", 8192, 8192, 8192, with_ref=False))  # profiler size
    cases.append(gemm_case("c5_gemm_128x64x256", 128, 64, 256))
    cases.append(gemm_case("c5_gemm_256x512x512", 256, 512, 512))
    cases.append(gemm_case("c5_gemm_384x1024x768", 384, 1024, 768))
    cases.append(gemm_case("c5_gemm_200x136x300", 200, 136, 300))
    # ragged CTA-pair tiles: last M tile holds 8 rows (its second CTA reads only
    # out-of-bounds rows), last N tile 136 of 256 columns, 5 k-blocks
    cases.append(gemm_case("c5_gemm_520x320x392", 520, 320, 392))
    # K not a multiple of the 64-wide k-block (the last block is half out of bounds), N ragged
    cases.append(gemm_case("c5_gemm_264x200x264", 264, 200, 264))
    # B stored [N, K] (K-major B): both tcgen05 kernels and the single-CTA one
    cases.append(gemm_case("c5_gemm_bnk_384x256x512", 384, 256, 512, b_nk=True))
    cases.append(gemm_case("c5_gemm_bnk_128x128x256", 128, 128, 256, b_nk=True))
    cases.append(gemm_case("m_matmul_f32_17x33x19", 17, 33, 19, dtype=F32, epilogue=False))
    cases.append(gemm_case("m_matmul_f32_64x64x64", 64, 64, 64, dtype=F32, epilogue=False))
    cases.append(gemm_case("m_matmul_f32_bias_96x160x80", 96, 160, 80, dtype=F32))
    # the reference generators' pointwise catalog
    for op, n in (("add", 333), ("subtract", 512), ("multiply", 768), ("maximum", 4096),
                  ("minimum", 256), ("divide", 200)):
        cases.append(binary_case(f"p_{op}_{n}", op, n))
    for op, n, pa in (("relu", 1000, None), ("exp", 256, None), ("tanh", 512, None),
                      ("sigmoid", 384, None), ("abs", 222, None), ("negative", 111, None),
                      ("sqrt", 256, 1e-6), ("rsqrt", 192, 1e-3), ("log", 160, 1e-3),
                      ("silu", 200, None), ("copy", 96, None), ("square", 300, None),
                      ("reciprocal", 130, None), ("exp2", 64, None), ("log2", 70, 1e-3)):
        cases.append(unary_case(f"p_{op}_{n}", op, n, prep_abs=pa))
    for which, n in (("relu_mul", 300), ("scale_shift", 1536), ("leaky", 180), ("clamp", 240),
                     ("where", 384), ("select", 256), ("cond_else", 300), ("square_scale", 512),
                     ("silu_sigmoid", 4100), ("exp_log_sqrt", 2051), ("contract_square_add", 1000),
                     ("contract_nonadjacent", 1000), ("contract_sub", 1000), ("contract_multiuse", 1000),
                     ("contract_log_add", 1000), ("contract_two_products", 1000), ("contract_cond", 1000),
                     ("contract_two_products_swapped", 1000)):
        cases.append(chain_case(f"p_{which}_{n}", n, which))
    # fused row reduction + pointwise epilogue (rmsnorm / softmax / l2norm)
    for kind in ("rmsnorm", "softmax", "l2norm"):
        cases.append(rownorm_case(f"f_{kind}_64x1000", 64, 1000, kind))
        cases.append(rownorm_case(f"f_{kind}_7x4096", 7, 4096, kind))
        cases.append(rownorm_case(f"f_{kind}_33x130", 33, 130, kind))
        cases.append(rownorm_case(f"f_{kind}_bench_16384x8192", 16384, 8192, kind, config=f"f_{kind}"))
    cases.append(rownorm_case("f_rmsnorm_bf16_64x1000", 64, 1000, "rmsnorm", dtype=BF16))
    cases.append(rownorm_case("f_softmax_bf16_33x4096", 33, 4096, "softmax", dtype=BF16))
    # naive attention (one thread per output cell, scores recomputed per pass)
    cases.append(attention_case("a_attn_64x32", 64, 32))
    cases.append(attention_case("a_attn_100x48", 100, 48))
    cases.append(attention_case("a_attn_256x64", 256, 64))
    cases.append(attention_case("a_attn_krows_80x40", 80, 40, k_rows=True))  # keys stored [seq, dim]
    cases.append(attention_case("a_attn_bench_2048x64", 2048, 64, config="a_attn"))
    cases.append(add2d_case("p_add2d_7x13", 7, 13))
    cases.append(add2d_case("p_add2d_32x64", 32, 64))
    cases.append(vec4_case("p_vec4_1024", 1024))
    cases.append(const_scale_case("p_const_scale_777", 777))
    cases.append(launch3d_case("p_launch3d_64"))
    # Emmy's cp.async shared-memory matmul schedule (the schedule family)
    cases.append(cpasync_matmul_case("s_cpasync_matmul_64x48x80", 64, 48, 80))
    cases.append(cpasync_matmul_case("s_cpasync16_matmul_32x64x48", 32, 64, 48, wide=True))
    cases.append(pre_carry_case("s_pre_carry_500", 500))
    cases.append(smem_matmul_case("s_smem_matmul_48x32x64", 48, 32, 64))
    cases.append(cond_load_case("p_cond_load_300", 300))
    cases.append(raster_matmul_case("s_raster_matmul_48x40x64", 48, 40, 64, 4))
    cases.append(aux_threads_case("s_aux_add_1000", 1000))
    cases.append(big_smem_case("s_bigsmem_reverse_6x16384", 6, 16384))
    cases.append(loose_statements_case("s_loose_nodes_32"))
    return cases


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    ap.add_argument("--only", default="", help="comma-separated case ids to (re)write; default all")
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.reference).resolve()))
    sys.dont_write_bytecode = True
    ref = importlib.import_module("compile")
    CASES.mkdir(parents=True, exist_ok=True)
    only = {c for c in args.only.split(",") if c}
    old = {}
    if only and (CASES / "INDEX.json").is_file():
        old = {r["id"]: r for r in json.loads((CASES / "INDEX.json").read_text())["cases"]}
    index = []
    for case in all_cases():
        if only and case.cid not in only and case.cid in old:
            index.append(old[case.cid])
            continue
        index.append(case.write(CASES, ref.compile_bundle))
    (CASES / "INDEX.json").write_text(json.dumps({"cases": index}, indent=1) + "\n")
    print(f"indexed {len(index)} cases under {CASES}", file=sys.stderr)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
