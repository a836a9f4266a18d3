"""Soundness of the staged-matmul proof (families/canon.py), CPU only.

Mutations of a cp.async-staged matmul's index expressions: the copy
sources, the shared-memory slots written and read, the output cell.  Whenever
the proof accepts a mutant, the oracle's lockstep evaluation of that mutant,
which follows the schedule as written, must equal the sequential-fma matmul
of the same inputs.  The proof may refuse correct mutants; it must never accept
a wrong one.
"""

from __future__ import annotations

import itertools
import sys

import numpy as np

from conftest import REPO

sys.path.insert(0, str(REPO / "oracle"))

TS, M, K, N = 8, 16, 16, 24


def _build(mut):
    """The staged matmul (8x8 tiles, 64-thread blocks) with mutation ``mut``
    applied, in the oracle's IR classes and in ours (same structure)."""
    from emmy import _core as E
    from emmy_ptx_compiler_b200 import ir as O

    def mk(ns):
        V, L = ns.Var, (lambda v: ns.Literal(v, "int"))
        add = lambda a, b: ns.BinaryExpr("+", a, b)  # noqa: E731
        mul = lambda a, c: ns.BinaryExpr("*", a, L(c))  # noqa: E731
        row = add(mul(V("bi"), mut["row_scale"]), V(mut["row_thread"]))
        col = add(mul(V("bj"), TS), V(mut["col_thread"]))
        a_src = (add(mul(V("bi"), TS), V("ty")), add(add(mul(V("kt"), mut["a_kt"]), V("tx")), L(mut["a_off"])))
        b_src = (add(mul(V("kt"), TS), V(mut["b_row_thread"])), add(mul(V("bj"), TS), V("tx")))
        sa_slot = (V("ty"), V("tx")) if not mut["swap_sa"] else (V("tx"), V("ty"))
        a_read = (V("ty"), V("kk")) if not mut["swap_ra"] else (V("kk"), V("ty"))
        f32 = ns.DataType("f32", np.dtype("float32"), 4) if ns is E else O.DataType("f32", "float32", 4)
        tile = ns.Tile(axes=(ns.Axis("bi", M // TS), ns.Axis("bj", N // TS), ns.Axis("ty", TS), ns.Axis("tx", TS)),
                       block_threads=TS * TS, body=(
            ns.Smem("As", (TS, TS), "float", 16), ns.Smem("Bs", (TS, TS), "float", 16),
            ns.Init("acc", 0.0, dtype=f32),
            ns.Loop(axis=ns.Axis("kt", K // TS), body=(
                ns.CpAsyncCopy("As", sa_slot, "A", a_src, 4),
                ns.CpAsyncCopy("Bs", (V("ty"), V("tx")), "B", b_src, 4),
                ns.CpAsyncCommit(), ns.CpAsyncWait(0), ns.Sync(),
                ns.Loop(axis=ns.Axis("kk", TS), body=(
                    ns.Load(names=("a",), input="As", index=a_read, dtype=f32),
                    ns.Load(names=("b",), input="Bs", index=(V("kk"), V("tx")), dtype=f32),
                    ns.Assign("p", ns.ElementwiseImpl("multiply"), ("a", "b"), f32),
                    ns.Accum("acc", "p", ns.ElementwiseImpl("add"), f32, axes=("kk",)))),
                ns.Sync())),
            ns.Write(output="C", index=(row, col), values=("acc",), value_dtype=f32)))
        return ns.KernelOp(name="k_mut", body=(tile,))
    return mk(E), mk(O)


CHOICES = {"row_scale": [TS, 4], "row_thread": ["ty", "tx"], "col_thread": ["tx", "ty"], "a_kt": [TS, 4],
           "a_off": [0, 1], "b_row_thread": ["ty", "tx"], "swap_sa": [False, True], "swap_ra": [False, True]}


def test_every_accepted_mutant_computes_the_matmul():
    """All 256 combinations of the mutations above."""
    import interp
    from emmy_ptx_compiler_b200.families import canon
    shapes = {"A": (M, K), "B": (K, N), "C": (M, N)}
    dtypes = {"A": "f32", "B": "f32", "C": "f32"}
    meta = {"grid": [(M // TS) * (N // TS), 1, 1], "block": [TS * TS, 1, 1]}
    rng = np.random.default_rng(0)
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = rng.standard_normal((K, N)).astype(np.float32)
    want = np.empty((M, N), np.float32)
    interp.lib().ora_gemm_seqfma_f32(interp._p(A), interp._p(B), interp._p(want), M, N, K, 0)
    accepted = []
    for combo in itertools.product(*CHOICES.values()):
        mut = dict(zip(CHOICES, combo))
        kop_oracle, kop_ours = _build(mut)
        if canon.staged_matmul(kop_ours, shapes, dtypes, meta) is None:
            continue
        accepted.append(mut)
        got = interp._eval_simt(kop_oracle, shapes, dtypes, {"A": A, "B": B}, {"C": (M, N)}, meta)["C"]
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), mut
    # the schedule itself, and the variant that transposes both the A slot written and the A slot read
    assert len(accepted) >= 2


def test_the_unmutated_schedule_is_accepted():
    from emmy_ptx_compiler_b200.families import canon
    base = {"row_scale": TS, "row_thread": "ty", "col_thread": "tx", "a_kt": TS, "a_off": 0, "b_row_thread": "ty",
            "swap_sa": False, "swap_ra": False}
    _, kop = _build(base)
    assert canon.staged_matmul(kop, {"A": (M, K), "B": (K, N), "C": (M, N)},
                               {"A": "f32", "B": "f32", "C": "f32"},
                               {"grid": [6, 1, 1], "block": [64, 1, 1]}) is not None
