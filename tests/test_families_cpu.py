"""Host-side checks of the family planners and the launch record (CPU only)."""

from __future__ import annotations

import json
import subprocess

import pytest

from conftest import CASES, REPO


def _plan_inputs(cid: str):
    from emmy_ptx_compiler_b200 import frontend
    ir_path = next((CASES / cid).glob("*.ir.json"))
    raw = json.loads(ir_path.read_text())
    info = frontend.load_graph(raw)
    mk = frontend.load_meta_kernel(ir_path, info.kop.name)
    shapes, dtypes = frontend.load_shapes(raw, info.kop, mk)
    return info.kop, shapes, dtypes, frontend.arg_order_for(info.kop, mk)


def test_launch_record_initialiser_matches_the_struct(tmp_path):
    """The Python-emitted aggregate initialiser fills the C struct field by
    field: compile it on the host against the header and read it back."""
    from emmy_ptx_compiler_b200.families.common import LaunchPlan, ParamSpec, TmapSpec, launch_record_source
    lp = LaunchPlan((7, 2, 1), (192, 1, 1), smem=197888, cluster=(2, 1, 1), fill_waves=3, grid_quantum=16,
                    range_total=12345, range_align=256, range_bytes=[8, 0, 4])
    params = [ParamSpec("a", "ptr", "bf16"), ParamSpec("s", "scalar", "f32"), ParamSpec("c", "ptr", "f32")]
    tm = TmapSpec(0, 9, [64, 128], [128], [64, 32], 3, 3)
    rec = launch_record_source("gemm", lp, params, [tm])
    prog = tmp_path / "rec.cpp"
    prog.write_text(
        "#define __device__\n#include <cstdio>\n#include <cstddef>\n" + rec + """
int main() {
    const EmmyLaunchRecord &r = emmy_launch_record;
    std::printf("%u %u %u %u %u %u %u %u %u %llu %u %llu %llu %llu %u %u\\n", r.family, r.flags, r.grid[0], r.grid[1],
                r.block[0], r.dyn_smem, r.nparams, r.param_kind[1], r.ntmaps,
                (unsigned long long)r.range_total, r.range_align, (unsigned long long)r.range_bytes[0],
                (unsigned long long)r.range_bytes[2], (unsigned long long)r.tmaps[0].dims[1], r.tmaps[0].box[1],
                r.grid_quantum);
    return 0;
}
""")
    exe = tmp_path / "rec"
    cc = subprocess.run(["g++", "-std=c++17", f"-I{REPO / 'include'}", str(prog), "-o", str(exe)],
                        capture_output=True, text=True)
    assert cc.returncode == 0, cc.stderr[-2000:]
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()
    # family 3 (gemm); flags = cluster 2 | FILL_GRID | RANGE; grid[0] carries the waves
    assert out == ["3", str(2 | 0x100 | 0x200), "3", "2", "192", "197888", "3", "1", "1",
                   "12345", "256", "8", "4", "128", "32", "16"]


def test_softmax_reuses_its_exp_across_passes():
    from emmy_ptx_compiler_b200.families import rownorm
    kop, shapes, dtypes, args = _plan_inputs("f_softmax_64x1000")
    plan = rownorm.match(kop, shapes, dtypes)
    keep, reuse = rownorm.reuse_plan(plan, {})
    assert keep == {(1, "e1"): 0}
    assert reuse == {(2, "e2"): 0}


def test_rmsnorm_has_nothing_to_reuse():
    """Its later pass multiplies (products are never reused: contraction
    depends on how each product is used)."""
    from emmy_ptx_compiler_b200.families import rownorm
    kop, shapes, dtypes, args = _plan_inputs("f_rmsnorm_64x1000")
    plan = rownorm.match(kop, shapes, dtypes)
    assert rownorm.reuse_plan(plan, {}) == ({}, {})


def test_row_fused_plan_streams_and_ranges():
    from emmy_ptx_compiler_b200.families import rownorm
    kop, shapes, dtypes, args = _plan_inputs("f_rmsnorm_64x1000")
    plan = rownorm.match(kop, shapes, dtypes)
    assert plan.streamed == ["x"] and plan.vectors == ["w"] and plan.outputs == ["y"]
    assert rownorm.range_bytes(plan, args, {}, dtypes, shapes) == [4000, 0, 4000]


def test_attention_plan_splits_row_and_cell_work():
    from emmy_ptx_compiler_b200.families import attention
    kop, shapes, dtypes, args = _plan_inputs("a_attn_64x32")
    plan = attention.match(kop, shapes, dtypes)
    loops = [s for s in plan.steps if isinstance(s, attention.KeyLoop)]
    assert len(loops) == 3 and plan.k_dk and plan.v == "v" and plan.cell_accs == ["acc"]
    assert [a for a, _ in loops[0].row_accs] == ["m"] and [a for a, _ in loops[1].row_accs] == ["den"]
    assert loops[2].stash == ["wt"] and not loops[2].row_accs


@pytest.mark.parametrize("cid,family", [("c3_rowsummax_64x5000", "reduction"), ("c2_gelu_64x1000", "pointwise"),
                                        ("c5_gemm_128x64x256", "gemm")])
def test_new_families_do_not_claim_other_kernels(cid, family):
    from emmy_ptx_compiler_b200.families import attention, rownorm
    kop, shapes, dtypes, args = _plan_inputs(cid)
    assert attention.match(kop, shapes, dtypes) is None
    assert rownorm.match(kop, shapes, dtypes) is None


# ------------------------------------------------------------------ schedule family


@pytest.mark.parametrize("cid,wide", [("s_cpasync_matmul_64x48x80", False), ("s_cpasync16_matmul_32x64x48", True)])
def test_cp_async_schedule_lowers_to_the_schedule_family(cid, wide):
    """A cp.async-staged matmul is proven a matmul and lowered by the GEMM
    family; forced to keep its own schedule, it keeps the reference's thread
    model and copy widths."""
    from emmy_ptx_compiler_b200 import compiler
    kop, shapes, dtypes, args = _plan_inputs(cid)
    meta = json.loads((CASES / cid / "meta.json").read_text())["kernels"][0]
    assert compiler.lower(kop, shapes, dtypes, args, meta).kernel.family == "gemm"
    low = compiler.lower(kop, shapes, dtypes, args, meta, {"family": "schedule"})
    ks = low.kernel
    assert ks.family == "schedule"
    assert ks.launch.grid == tuple(meta["grid"]) and ks.launch.block == tuple(meta["block"])
    src = ks.source
    assert "cp.async.cg.shared.global" in src if wide else "cp.async.ca.shared.global" in src
    assert "cp.async.commit_group" in src and "cp.async.wait_group 0" in src
    assert "__syncthreads();" in src and "__shared__" in src


@pytest.mark.parametrize("cid", ["c3_rowsummax_5x64", "r_mean_777", "r_atomic_zp_sum_128", "f_softmax_33x130",
                                 "a_attn_64x32", "m_matmul_f32_17x33x19", "p_launch3d_64", "p_select_256"])
def test_every_family_input_also_lowers_as_its_own_schedule(cid):
    """The schedule family accepts what the fast families accept (the GPU test
    compares its outputs with the reference PTX bit for bit)."""
    from emmy_ptx_compiler_b200 import compiler
    ir_path = next((CASES / cid).glob("*.ir.json"))
    b = compiler.compile_bundle(ir_path, want_cubin=True, options={"family": "schedule"})
    assert b["family"] == "schedule" and len(b["cubin"]) > 0


def test_tensor_core_nodes_are_reported_not_lowered():
    """sm_90 tensor-core nodes (here mma.sync fragments) have no sm_100a
    lowering in any family: the compiler names them."""
    from emmy_ptx_compiler_b200 import compiler, ir
    from emmy_ptx_compiler_b200.errors import UnsupportedIR
    f16 = ir.DataType("f16", None, 2)
    body = (ir.Tile(axes=(ir.Axis("a0", 32),), body=(
        ir.RegFragment("fa", "a", (16, 8, 16), f16, 4),
        ir.MmaSyncPtx("fc", "fa", "fb", (16, 8, 16), "f16", "f32"),
    )),)
    kop = ir.KernelOp(name="k_mma", body=body)
    with pytest.raises(UnsupportedIR, match="MmaSyncPtx"):
        compiler.lower(kop, {"x": (32,)}, {"x": "f32"}, ["x"], {"grid": [1, 1, 1], "block": [32, 1, 1]})


def _staged_matmul_kop(m=64, k=48, n=80, *, b_src=None, second_sync=True, a_kt_shift=16, wide_cols=4):
    """The cp.async-staged matmul of the s_cpasync fixtures, with knobs that break it."""
    from emmy_ptx_compiler_b200 import ir
    F32 = ir.DataType("f32", "float32", 4)
    ts = 16
    V, L = ir.Var, lambda v: ir.Literal(v, "int")  # noqa: E731
    add, mul = (lambda a, b: ir.BinaryExpr("+", a, b)), (lambda a, b: ir.BinaryExpr("*", a, b))  # noqa: E731
    row, col = add(mul(V("bi"), L(ts)), V("ty")), add(mul(V("bj"), L(ts)), V("tx"))
    tx4 = mul(V("tx"), L(4))
    a_src = (row, add(mul(V("kt"), L(a_kt_shift)), tx4))
    b_src = b_src or (add(mul(V("kt"), L(ts)), V("ty")), add(mul(V("bj"), L(ts)), tx4))
    copies = (ir.Cond(ir.BinaryExpr("<", V("tx"), L(wide_cols)), body=(
        ir.CpAsyncCopy("As", (V("ty"), tx4), "A", a_src, 16),
        ir.CpAsyncCopy("Bs", (V("ty"), tx4), "B", b_src, 16),
    )),)
    kt_body = (*copies, ir.CpAsyncCommit(), ir.CpAsyncWait(0), ir.Sync(),
               ir.Loop(axis=ir.Axis("kk", ts), body=(
                   ir.Load(names=("a",), input="As", index=(V("ty"), V("kk")), dtype=F32),
                   ir.Load(names=("b",), input="Bs", index=(V("kk"), V("tx")), dtype=F32),
                   ir.Assign("p", ir.ElementwiseImpl("multiply"), ("a", "b"), F32),
                   ir.Accum("acc", "p", ir.ElementwiseImpl("add"), F32, axes=("kk",)))))
    if second_sync:
        kt_body += (ir.Sync(),)
    tile = ir.Tile(axes=(ir.Axis("bi", m // ts), ir.Axis("bj", n // ts), ir.Axis("ty", ts), ir.Axis("tx", ts)),
                   block_threads=ts * ts, body=(
        ir.Smem("As", (ts, ts), "float", 16), ir.Smem("Bs", (ts, ts), "float", 16),
        ir.Init("acc", 0.0, dtype=F32),
        ir.Loop(axis=ir.Axis("kt", k // ts), body=kt_body),
        ir.Write(output="C", index=(row, col), values=("acc",), value_dtype=F32)))
    kop = ir.KernelOp(name="k_staged", body=(tile,))
    shapes = {"A": (m, k), "B": (k, n), "C": (m, n)}
    return kop, shapes, {"A": "f32", "B": "f32", "C": "f32"}


def test_staged_matmul_is_proven_and_lowered_as_a_gemm():
    from emmy_ptx_compiler_b200 import compiler
    from emmy_ptx_compiler_b200.families import canon
    kop, shapes, dtypes = _staged_matmul_kop()
    meta = {"grid": [20, 1, 1], "block": [256, 1, 1]}
    naive = canon.staged_matmul(kop, shapes, dtypes, meta)
    assert naive is not None
    low = compiler.lower(kop, shapes, dtypes, ["A", "B", "C"], meta)
    assert low.kernel.family == "gemm" and low.kernel.notes.get("canonical_form")


@pytest.mark.parametrize("knob", ["b_transposed", "no_second_sync", "wrong_k_shift", "missing_copies"])
def test_near_miss_schedules_keep_their_own_schedule(knob):
    """A staged matmul the proof cannot establish stays in the schedule family."""
    from emmy_ptx_compiler_b200 import compiler, ir
    from emmy_ptx_compiler_b200.families import canon
    V, L = ir.Var, lambda v: ir.Literal(v, "int")  # noqa: E731
    kw = {}
    if knob == "b_transposed":
        tx4 = ir.BinaryExpr("*", V("tx"), L(4))
        kw["b_src"] = (ir.BinaryExpr("+", ir.BinaryExpr("*", V("bj"), L(16)), tx4),
                       ir.BinaryExpr("+", ir.BinaryExpr("*", V("kt"), L(16)), V("ty")))
    elif knob == "no_second_sync":
        kw["second_sync"] = False
    elif knob == "wrong_k_shift":
        kw["a_kt_shift"] = 8
    else:
        kw["wide_cols"] = 3
    # square operands for the transposed copy, so only the index proof can tell
    kop, shapes, dtypes = _staged_matmul_kop(m=64, k=64, n=64, **kw) if knob == "b_transposed" \
        else _staged_matmul_kop(**kw)
    meta = {"grid": [20, 1, 1], "block": [256, 1, 1]}
    assert canon.staged_matmul(kop, shapes, dtypes, meta) is None
    low = compiler.lower(kop, shapes, dtypes, ["A", "B", "C"], meta)
    assert low.kernel.family == "schedule"


def _plain_copy_kop(swap: bool):
    """The s_smem_matmul fixture's schedule; ``swap`` stores each loaded element into the other buffer."""
    from emmy_ptx_compiler_b200 import ir
    F32 = ir.DataType("f32", "float32", 4)
    ts, m, k, n = 16, 48, 32, 48
    V, L = ir.Var, lambda v: ir.Literal(v, "int")  # noqa: E731
    at = lambda blk, thr: ir.BinaryExpr("+", ir.BinaryExpr("*", V(blk), L(ts)), thr)  # noqa: E731
    row, col = at("bi", V("ty")), at("bj", V("tx"))
    sa, sb = ("Bs", "As") if swap else ("As", "Bs")
    tile = ir.Tile(axes=(ir.Axis("bi", m // ts), ir.Axis("bj", n // ts), ir.Axis("ty", ts), ir.Axis("tx", ts)),
                   block_threads=ts * ts, body=(
        ir.Smem("As", (ts, ts), "float", 16), ir.Smem("Bs", (ts, ts), "float", 16),
        ir.Init("acc", 0.0, dtype=F32),
        ir.Loop(axis=ir.Axis("kt", k // ts), body=(
            ir.Load(names=("ga",), input="A", index=(row, at("kt", V("tx"))), dtype=F32),
            ir.Write(output=sa, index=(V("ty"), V("tx")), values=("ga",), value_dtype=F32),
            ir.Load(names=("gb",), input="B", index=(at("kt", V("ty")), col), dtype=F32),
            ir.Write(output=sb, index=(V("ty"), V("tx")), values=("gb",), value_dtype=F32),
            ir.Sync(),
            ir.Loop(axis=ir.Axis("kk", ts), body=(
                ir.Load(names=("a",), input="As", index=(V("ty"), V("kk")), dtype=F32),
                ir.Load(names=("b",), input="Bs", index=(V("kk"), V("tx")), dtype=F32),
                ir.Assign("p", ir.ElementwiseImpl("multiply"), ("a", "b"), F32),
                ir.Accum("acc", "p", ir.ElementwiseImpl("add"), F32, axes=("kk",)))),
            ir.Sync())),
        ir.Write(output="C", index=(row, col), values=("acc",), value_dtype=F32)))
    return (ir.KernelOp(name="k_plain", body=(tile,)), {"A": (m, k), "B": (k, n), "C": (m, n)},
            {"A": "f32", "B": "f32", "C": "f32"})


@pytest.mark.parametrize("swap", [False, True])
def test_plain_copy_staging_is_proven_only_when_right(swap):
    from emmy_ptx_compiler_b200.families import canon
    kop, shapes, dtypes = _plain_copy_kop(swap)
    got = canon.staged_matmul(kop, shapes, dtypes, {"block": [256, 1, 1]})
    assert (got is None) == swap


@pytest.mark.parametrize("cid, mode", [("f_rmsnorm_bench_16384x8192", "cta"), ("f_softmax_bench_16384x8192", "cta"),
                                       ("f_l2norm_7x4096", "cta"), ("f_rmsnorm_64x1000", "warp"),
                                       ("f_softmax_64x1000", "warp"), ("f_rmsnorm_33x130", "persistent"),
                                       ("f_softmax_bf16_33x4096", "persistent")])
def test_row_fused_grid_follows_the_row_range(cid, mode):
    """Rows of 16 KiB or more get one CTA each; rows that fit a warp's registers
    one warp each, 8 rows per CTA.  Both records ask for EMMY_LR_GRID_UNITS
    (grid_quantum = rows per CTA), so that a range launch sizes its grid from
    its rows.  Other rows (unaligned widths, too few rows) keep the
    occupancy-filled or fixed grid."""
    from emmy_ptx_compiler_b200.families import rownorm
    from emmy_ptx_compiler_b200.families.common import FLAG_GRID_UNITS, launch_record_source
    kop, shapes, dtypes, args = _plan_inputs(cid)
    plan = rownorm.match(kop, shapes, dtypes)
    ks = rownorm.generate(kop, plan, shapes, dtypes, args, {}, set(plan.outputs))
    assert ks.notes["cta_per_row"] is (mode == "cta")
    assert ks.notes["warp_per_row"] is (mode == "warp")
    rec = launch_record_source("rownorm", ks.launch, ks.params)
    flags = int(rec.split("EMMY_LR_VERSION, 4u, ")[1].split("u")[0])
    assert bool(flags & FLAG_GRID_UNITS) is (mode != "persistent")
    if mode == "cta":
        assert ks.launch.grid[0] == plan.rows and ks.launch.grid_quantum == 1 and not ks.launch.fill_waves
    if mode == "warp":
        assert ks.launch.block[0] == 32 * rownorm.WR_ROWS and ks.notes["threads_per_row"] == 32
        assert ks.launch.grid[0] == -(-plan.rows // ks.launch.grid_quantum)
        assert "__syncthreads" not in ks.source.split("emmy_launch_record")[0].split("__launch_bounds__")[1]


def test_attention_exchange_choice_and_launch_record():
    """The bench shape (16 query tiles x 8 CTAs = 128 CTAs) fits on the SMs at
    once, so "auto" takes the grid exchange: no cluster, a cooperative launch,
    enough shared memory that no SM holds two of these CTAs (each takes all
    512 tensor-memory columns), and a drop-in that never runs the fast body."""
    from emmy_ptx_compiler_b200 import compiler
    from emmy_ptx_compiler_b200.families import attention, attention_tc
    from emmy_ptx_compiler_b200.families.common import FLAG_COOPERATIVE, launch_record_source
    kop, shapes, dtypes, args = _plan_inputs("a_attn_bench_2048x64")
    plan = attention.match(kop, shapes, dtypes)
    lay, why = attention_tc.layout(plan, shapes, dtypes)
    assert lay["XM"] == "grid" and lay["CL"] == 8 and lay["TCOLS"] == 512
    assert lay["SMEM_LAUNCH"] > attention_tc.SM_SMEM_BYTES // 2 - 1024
    cl, _ = attention_tc.layout(plan, shapes, dtypes, exchange="cluster")
    assert cl["XM"] == "cluster"
    ks = attention_tc.generate_tc(kop, plan, lay, shapes, dtypes, args, {}, {plan.out_name})
    assert ks.launch.cooperative and ks.launch.cluster == (1, 1, 1)
    rec = launch_record_source("attention", ks.launch, ks.params)
    flags = int(rec.split("EMMY_LR_VERSION, 5u, ")[1].split("u")[0])
    assert flags & FLAG_COOPERATIVE and (flags & 0xFF) == 1
    b = compiler.compile_bundle(next((CASES / "a_attn_bench_2048x64").glob("*.ir.json")))
    assert b["notes"]["exchange"] == "grid"
    assert b["notes"]["entries"]["drop_in_path"].startswith("the IR's own schedule under every launch")


def test_attention_small_problems_keep_the_cluster_exchange():
    """Two query tiles: both exchanges fit, and the cluster's is the faster."""
    from emmy_ptx_compiler_b200.families import attention, attention_tc
    kop, shapes, dtypes, args = _plan_inputs("a_attn_256x64")
    plan = attention.match(kop, shapes, dtypes)
    lay, why = attention_tc.layout(plan, shapes, dtypes)
    assert lay["XM"] == "cluster" and lay["nq"] == 2
    lay, why = attention_tc.layout(plan, shapes, dtypes, exchange="grid")
    assert lay["XM"] == "grid"


def test_attention_grid_exchange_needs_every_cta_resident():
    from emmy_ptx_compiler_b200.families import attention, attention_tc
    kop, shapes, dtypes, args = _plan_inputs("a_attn_bench_2048x64")
    plan = attention.match(kop, shapes, dtypes)
    plan.SQ = 128 * 40               # 40 query tiles x 8 CTAs: more CTAs than SMs
    lay, why = attention_tc.layout(plan, shapes, dtypes)
    assert lay["XM"] == "cluster"
    lay, why = attention_tc.layout(plan, shapes, dtypes, exchange="grid")
    assert lay is None and "do not fit" in why[-1]


def test_pointwise_tune_option_changes_the_schedule_only():
    """``pointwise_tune`` sets the pointwise generator's unroll / pipelining /
    occupancy knobs; unknown keys are rejected."""
    from emmy_ptx_compiler_b200 import compiler
    ir_path = next((CASES / "c2_gelu_64x1000").glob("*.ir.json"))
    base = compiler.compile_bundle(ir_path)
    tuned = compiler.compile_bundle(ir_path, options={"pointwise_tune": {"unroll": 4, "pipeline": False,
                                                                         "min_blocks": 3}})
    assert tuned["family"] == base["family"] == "pointwise"
    assert "__launch_bounds__(256, 3)" in tuned["source"] and tuned["source"] != base["source"]
    with pytest.raises(ValueError):
        compiler.compile_bundle(ir_path, options={"pointwise_tune": {"unrol": 4}})


def test_cooperative_attention_without_a_schedule_still_compiles(monkeypatch):
    """When the IR's own schedule cannot be lowered, a cooperative attention
    module's drop-in entry only reports EMMY_STATUS_BAD_LAUNCH (a kernel cannot
    tell whether it was launched cooperatively); the fast entry is unchanged."""
    from emmy_ptx_compiler_b200 import compiler
    from emmy_ptx_compiler_b200.families import schedule
    monkeypatch.setattr(schedule, "match", lambda *a, **k: None)
    b = compiler.compile_bundle(next((CASES / "a_attn_bench_2048x64").glob("*.ir.json")), want_cubin=True)
    assert b["family"] == "attention" and b["notes"]["exchange"] == "grid"
    assert b["notes"]["entries"]["drop_in_path"].startswith("reports EMMY_STATUS_BAD_LAUNCH")
    assert b["cubin"][:4] == b"\x7fELF"


def test_reduction_chunking_rule():
    """Rows of two MIN_CHUNKs or more split in two chunks from half a wave of
    rows up; a full-array reduction splits into one chunk per CTA slot; short
    rows stay whole."""
    from emmy_ptx_compiler_b200.families import reduction
    assert reduction._pick_chunks(8192, 65536) == (2, 32768)     # C3
    assert reduction._pick_chunks(1024, 65536) == (2, 32768)     # C3's 8-GPU shard
    assert reduction._pick_chunks(65536, 4096) == (1, 4096)      # rows too short to split
    ch, length = reduction._pick_chunks(1, 1 << 31)              # C4
    assert ch == 1184 and ch * length >= 1 << 31 and length % 128 == 0


def test_pointwise_tiles_size_the_grid_from_the_range():
    """The vector path runs one CTA per 4 x 256 float4 tile: the record asks for
    EMMY_LR_GRID_UNITS with 4096 cells per CTA (a range launch gets one CTA per
    tile of its range), 256-thread blocks, and no occupancy fill."""
    from emmy_ptx_compiler_b200 import compiler
    from emmy_ptx_compiler_b200.families.common import FLAG_GRID_UNITS
    b = compiler.compile_bundle(next((CASES / "c2_gelu_full").glob("*.ir.json")))
    assert b["notes"]["order"] == "tile"
    assert b["launch"]["block"] == [256, 1, 1] and b["launch"]["grid"][0] == (1 << 28) // 4096
    flags = int(b["source"].split("EMMY_LR_VERSION, 1u, ")[1].split("u")[0])
    assert flags & FLAG_GRID_UNITS and not flags & 0x100
    assert "4096u," in b["source"].split("emmy_launch_record = {")[1]


def test_launch_record_flags_match_the_header():
    """The flag bits the Python side emits are the ones the C header defines."""
    import re
    from emmy_ptx_compiler_b200.families import common
    hdr = (REPO / "include" / "emmy_launch_record.h").read_text()
    defs = {m.group(1): int(m.group(2), 16) for m in re.finditer(r"#define EMMY_LR_(\w+) 0x([0-9A-Fa-f]+)u", hdr)}
    assert defs["FILL_GRID"] == common.FLAG_FILL_GRID
    assert defs["RANGE"] == common.FLAG_RANGE
    assert defs["GRID_UNITS"] == common.FLAG_GRID_UNITS
    assert defs["COOPERATIVE"] == common.FLAG_COOPERATIVE
    flags = [common.FLAG_FILL_GRID, common.FLAG_RANGE, common.FLAG_GRID_UNITS, common.FLAG_COOPERATIVE]
    assert all(f & 0xFF == 0 for f in flags) and len(set(flags)) == len(flags)   # clear of the cluster-size byte
