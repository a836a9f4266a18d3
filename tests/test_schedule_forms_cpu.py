"""The schedule family on IR forms the fixtures use rarely (CPU only): each
lowers, builds for sm_100a, and the oracle's lockstep evaluation runs it."""

from __future__ import annotations

import numpy as np
import pytest

from emmy_ptx_compiler_b200 import ir

F32 = ir.DataType("f32", "float32", 4)
V, L = ir.Var, (lambda v: ir.Literal(v, "int"))
EW = ir.ElementwiseImpl


def _bin(op, a, b):
    return ir.BinaryExpr(op, a, b)


def _loop_cond_select(n=256):
    """A Loop holding a Cond with an else branch, a Select, and a Let whose
    index uses a TernaryExpr and a CastExpr."""
    body = ir.Tile(axes=(ir.Axis("a0", n),), block_threads=128, body=(
        ir.Init("acc", 0.0, dtype=F32),
        ir.Loop(axis=ir.Axis("k", 4), body=(
            ir.Let("j", ir.TernaryExpr(_bin("<", V("k"), L(2)), _bin("+", V("a0"), V("k")),
                                       ir.CastExpr(_bin("-", V("a0"), V("k")), "i32")), "i32"),
            ir.Let("jc", ir.TernaryExpr(_bin("<", V("j"), L(0)), L(0),
                                        ir.TernaryExpr(_bin(">=", V("j"), L(n)), L(n - 1), V("j"))), "i32"),
            ir.Load(names=("x",), input="x", index=(V("jc"),), dtype=F32),
            ir.Cond(_bin(">", V("k"), L(1)), body=(
                ir.Assign("t", EW("multiply"), ("x", "x"), F32),
            ), else_body=(
                ir.Assign("t", EW("add"), ("x", "x"), F32),
            )),
            ir.Select("u", (ir.SelectBranch("t", _bin("<", V("k"), L(3))), ir.SelectBranch("x", L(1)))),
            ir.Accum("acc", "u", EW("add"), F32, axes=("k",)),
        )),
        ir.Write(output="y", index=(V("a0"),), values=("acc",), value_dtype=F32),
    ))
    return body, {"x": (n,), "y": (n,)}, {"grid": [n // 128, 1, 1], "block": [128, 1, 1]}


def _strided_barriers(n=512):
    """A seeded StridedLoop with an end expression, a named barrier with a
    count, a warp barrier and a shared buffer written then read across lanes."""
    body = ir.Tile(axes=(ir.Axis("b", n // 128), ir.Axis("t", 128)), block_threads=128, body=(
        ir.Smem("buf", (128,), "float", 16),
        ir.StridedLoop(axis=ir.Axis("e", n), start=V("t"), step=L(128), end=L(128), seed=True, body=(
            ir.Load(names=("v",), input="x", index=(_bin("+", _bin("*", V("b"), L(128)), V("e")),), dtype=F32),
            ir.Accum("s", "v", EW("add"), F32, axes=("e",)),
        )),
        ir.Write(output="buf", index=(V("t"),), values=("s",), value_dtype=F32),
        ir.Sync(barrier_id=1, count=128),
        ir.Sync(warp=True),
        ir.Load(names=("w",), input="buf", index=(_bin("-", L(127), V("t")),), dtype=F32),
        ir.Write(output="y", index=(_bin("+", _bin("*", V("b"), L(128)), V("t")),), values=("w",),
                 value_dtype=F32),
    ))
    return body, {"x": (n,), "y": (n,)}, {"grid": [n // 128, 1, 1], "block": [128, 1, 1]}


def _tree_inner(rows=4):
    """TreeHalve with an inner (index, scale): four independent 32-slot trees
    interleaved in one shared buffer, one per column."""
    cols = 4
    body = ir.Tile(axes=(ir.Axis("r", rows), ir.Axis("t", 128)), block_threads=128, body=(
        ir.Smem("sb", (128,), "float", 16),
        ir.Let("lane32", _bin("%", V("t"), L(32)), "i32"),
        ir.Let("col", _bin("/", V("t"), L(32)), "i32"),
        ir.Load(names=("v",), input="x", index=(_bin("+", _bin("*", V("r"), L(128)), V("t")),), dtype=F32),
        ir.Write(output="sb", index=(_bin("+", _bin("*", V("lane32"), L(cols)), V("col")),), values=("v",),
                 value_dtype=F32),
        ir.Sync(),
        ir.TreeHalve(bufs=("sb",), state=("acc",), state_b=("acc_o",),
                     combine_states=(ir.Assign("acc", EW("add"), ("acc", "acc_o")),),
                     length=32, tid_var="lane32", inner=("col", cols)),
        ir.Cond(_bin("==", V("lane32"), L(0)), body=(
            ir.Write(output="y", index=(_bin("+", _bin("*", V("r"), L(cols)), V("col")),), values=("acc",),
                     value_dtype=F32),
        )),
    ))
    return body, {"x": (rows * 128,), "y": (rows * cols,)}, {"grid": [rows, 1, 1], "block": [128, 1, 1]}


def _block3d(n=256):
    """A 3-D block (16 x 4 x 2) read through thread builtins."""
    body = ir.Tile(axes=(ir.Axis("a0", n),), block_threads=128, body=(
        ir.Let("ty", ir.Builtin("threadIdx.y"), "i32"),
        ir.Load(names=("v",), input="x", index=(V("a0"),), dtype=F32),
        ir.Let("fy", ir.CastExpr(V("ty"), "f32"), "f32"),
        ir.Assign("w", EW("add"), ("v", "fy"), F32),
        ir.Write(output="y", index=(V("a0"),), values=("w",), value_dtype=F32),
    ))
    return body, {"x": (n,), "y": (n,)}, {"grid": [n // 128, 1, 1], "block": [16, 4, 2]}


FORMS = {"loop_cond_select": _loop_cond_select, "strided_barriers": _strided_barriers,
         "tree_inner": _tree_inner, "block3d": _block3d}


@pytest.mark.parametrize("form", sorted(FORMS))
def test_schedule_form_builds(form):
    from emmy_ptx_compiler_b200.compiler import Compiler
    tile, shapes, meta = FORMS[form]()
    kop = ir.KernelOp(name=f"k_{form}", body=(tile,))
    c = Compiler(kop, shapes, {k: "f32" for k in shapes}, list(shapes), meta, options={"family": "schedule"})
    assert c.lower().kernel.family == "schedule"
    assert len(c.cubin()) > 0


def test_tree_with_inner_stride_in_the_oracle():
    """The lockstep oracle on the interleaved trees: each column's 32 values summed
    by halving (the tree order), compared with the same order in numpy."""
    import sys
    from conftest import REPO
    sys.path.insert(0, str(REPO / "oracle"))
    import interp
    from emmy._core import (Assign, Axis, BinaryExpr, Cond, ElementwiseImpl, KernelOp, Let, Literal, Load,
                            Smem, Sync, Tile, TreeHalve, Var, Write)
    rows, cols = 4, 4
    sh = {"x": (rows * 128,), "y": (rows * cols,)}
    lt = lambda v: Literal(v, "int")  # noqa: E731
    tile = Tile(axes=(Axis("r", rows), Axis("t", 128)), body=(
        Smem("sb", (128,), "float", 16),
        Let("lane32", BinaryExpr("%", Var("t"), lt(32)), "i32"),
        Let("col", BinaryExpr("/", Var("t"), lt(32)), "i32"),
        Load(names=("v",), input="x", index=(BinaryExpr("+", BinaryExpr("*", Var("r"), lt(128)), Var("t")),),
             dtype=None),
        Write(output="sb", index=(BinaryExpr("+", BinaryExpr("*", Var("lane32"), lt(cols)), Var("col")),),
              values=("v",), value_dtype=None),
        Sync(),
        TreeHalve(bufs=("sb",), state=("acc",), state_b=("acc_o",),
                  combine_states=(Assign("acc", ElementwiseImpl("add"), ("acc", "acc_o"), None),),
                  length=32, tid_var="lane32", inner=("col", cols)),
        Cond(BinaryExpr("==", Var("lane32"), lt(0)), body=(
            Write(output="y", index=(BinaryExpr("+", BinaryExpr("*", Var("r"), lt(cols)), Var("col")),),
                  values=("acc",), value_dtype=None),
        )),
    ), block_threads=128)
    x = np.random.default_rng(0).standard_normal(rows * 128).astype(np.float32)
    out = interp._eval_simt(KernelOp(name="k", body=(tile,)), sh, {"x": "f32", "y": "f32"}, {"x": x},
                            {"y": (rows * cols,)}, {"grid": [rows, 1, 1], "block": [128, 1, 1]})["y"]
    want = np.empty(rows * cols, np.float32)
    for r in range(rows):
        for c in range(cols):
            v = x[r * 128 + c * 32: r * 128 + c * 32 + 32].astype(np.float32).copy()
            step = 16
            while step:
                v[:step] = (v[:step] + v[step:2 * step]).astype(np.float32)
                step //= 2
            want[r * cols + c] = v[0]
    assert np.array_equal(out.view(np.uint32), want.view(np.uint32)), (out, want)
