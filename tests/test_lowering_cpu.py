"""Lowering: every fixture lands in the right kernel family and compiles for sm_100a (CPU only)."""

from __future__ import annotations

import subprocess

import pytest

from conftest import CASES, case_index


@pytest.fixture(scope="module")
def assembled(tmp_path_factory):
    """ptxas -arch=sm_100a on every fixture's printed module, run in parallel:
    case id -> (return code, stderr)."""
    import os
    from concurrent.futures import ThreadPoolExecutor
    from emmy_ptx_compiler_b200 import compiler
    root = tmp_path_factory.mktemp("ptxas")

    def one(rec):
        b = compiler.compile_bundle(CASES / rec["ir"])
        d = root / rec["id"]
        d.mkdir()
        (d / "m.ptx").write_text(b["ptx"])
        v = subprocess.run(["ptxas", "-arch=sm_100a", "-v", "-o", str(d / "m.cubin"), str(d / "m.ptx")],
                           capture_output=True, text=True)
        return rec["id"], (v.returncode, v.stderr)

    with ThreadPoolExecutor(max(1, min(16, os.cpu_count() or 1))) as ex:
        return dict(ex.map(one, case_index()))


@pytest.mark.parametrize("rec", case_index(), ids=lambda r: r["id"])
def test_family_and_build(rec, assembled):
    from emmy_ptx_compiler_b200 import compiler
    b = compiler.compile_bundle(CASES / rec["ir"], want_cubin=True)
    assert b["family"] == rec["family"], (rec["id"], b["family"])
    assert b["entry"] == rec["entry"]
    assert [p["name"] for p in b["params"]] == b["args"]
    assert b["cubin"][:4] == b"\x7fELF"
    # the printed module assembles for sm_100a and exports the KernelOp's entry
    rc, err = assembled[rec["id"]]
    assert rc == 0, err[-2000:]
    assert f"Compiling entry function '{rec['entry']}' for 'sm_100a'" in err


def test_headline_configs_take_the_fast_paths():
    from emmy_ptx_compiler_b200 import compiler
    c2 = compiler.compile_bundle(CASES / "c2_gelu_full" / "k_gelu_tanh_affine.ir.json")
    assert c2["notes"]["vector"] is True
    c3 = compiler.compile_bundle(CASES / "c3_rowsummax_full" / "k_row_sum_max_reduce.ir.json")
    assert c3["notes"]["vector"] and c3["notes"]["chunks"] == 2
    c4 = compiler.compile_bundle(CASES / "c4_sum_full" / "k_sum_1_reduce.ir.json")
    assert c4["notes"]["vector"] and c4["notes"]["chunks"] >= 148


def test_gelu_contracts_where_the_reference_does():
    """x*s+t and z3*c0+z become fma.rn (compile.py:1285-1303); the other
    products stay separate IEEE multiplies."""
    from emmy_ptx_compiler_b200 import compiler
    src = compiler.compile_bundle(CASES / "c2_gelu_64x1000" / "k_gelu_tanh_affine.ir.json")["source"]
    lane = src.split("{", 3)[-1]
    assert src.count("__fmaf_rn(") >= 2
    assert "emmy_tanh_ref(" in src
    assert "__fmul_rn(v_z, v_z)" in src and "__fmul_rn(v_z2, v_z)" in src
    del lane


def test_block_cooperative_kernel_keeps_its_schedule():
    """A Tile with a barrier is no pointwise kernel: it lowers as its own schedule."""
    from emmy_ptx_compiler_b200 import ir
    from emmy_ptx_compiler_b200.compiler import Compiler
    body = ir.Tile(axes=(ir.Axis("a0", ir.Dim(32)),), body=(
        ir.Load(names=("v",), input="x", index=(ir.Var("a0"),)),
        ir.Sync(),
        ir.Write(output="y", index=(ir.Var("a0"),), values=("v",)),
    ))
    kop = ir.KernelOp(name="k_sync", body=(body,))
    low = Compiler(kop, {"x": (32,), "y": (32,)}, {"x": "f32", "y": "f32"}, ["x", "y"]).lower()
    assert low.kernel.family == "schedule" and "__syncthreads();" in low.kernel.source


def test_unsupported_kernel_is_reported():
    from emmy_ptx_compiler_b200 import ir
    from emmy_ptx_compiler_b200.compiler import Compiler
    from emmy_ptx_compiler_b200.errors import UnsupportedIR
    body = ir.Tile(axes=(ir.Axis("a0", ir.Dim(32)),), body=(
        ir.TmaLoad("smem_a", (ir.Literal(0, "int"),), "tensormap", (ir.Literal(0, "int"),), "mbar0"),
        ir.Load(names=("v",), input="x", index=(ir.Var("a0"),)),
        ir.Write(output="y", index=(ir.Var("a0"),), values=("v",)),
    ))
    kop = ir.KernelOp(name="k_bad", body=(body,))
    with pytest.raises(UnsupportedIR, match="TmaLoad"):
        Compiler(kop, {"x": (32,), "y": (32,)}, {"x": "f32", "y": "f32"}, ["x", "y"]).lower()


def test_python_ir_api_matches_reference_constructor_style():
    """IR built in Python (as the reference's tests build it) compiles."""
    from emmy_ptx_compiler_b200 import ir
    from emmy_ptx_compiler_b200.compiler import Compiler
    F32 = ir.DataType("f32", "float32", 4)
    tile = ir.Tile(axes=(ir.Axis("a0", ir.Dim(100)),), block_threads=128, body=(
        ir.Load(names=("in0",), input="x", index=(ir.Var("a0"),), dtype=F32),
        ir.Assign(name="r", op=ir.ElementwiseImpl("sigmoid"), args=("in0",), dtype=F32),
        ir.Write(output="y", index=(ir.Var("a0"),), values=("r",), value_dtype=F32),
    ))
    kop = ir.KernelOp(name="k_sig", body=(tile,))
    c = Compiler(kop, {"x": (100,), "y": (100,)}, {"x": "f32", "y": "f32"}, ["x", "y"],
                 {"block": [128, 1, 1], "grid": [1, 1, 1]})
    assert c.lower().kernel.family == "pointwise"
    assert c.run().isascii()


def test_bundle_reports_register_counts_per_entry():
    """compile_bundle's ``virt_regs`` (compile.py:3194-3215 reports its virtual
    registers) carries ptxas's per-entry register and spill counts for sm_100a:
    the drop-in entry and, where there is one, the fast ``__emmy`` twin."""
    from emmy_ptx_compiler_b200 import compiler
    from conftest import CASES
    b = compiler.compile_bundle(next((CASES / "c5_gemm_200x136x300").glob("*.ir.json")))
    regs = b["virt_regs"]
    assert regs["registers"] > 0 and regs["spill_stores"] == 0
    assert set(regs["entries"]) == {b["entry"], b["entry"] + "__emmy"}
    assert all(e["registers"] <= 255 for e in regs["entries"].values())
