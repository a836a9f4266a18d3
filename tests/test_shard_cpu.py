"""Sharding a KernelOp over GPUs (emmy_ptx_compiler_b200.shard), on CPU.

The shard IRs are evaluated by the CPU oracle on the matching slices of the
inputs: for a row split the concatenated shard outputs must equal the whole
KernelOp's output bit for bit (rows are independent and each shard runs the
same per-row code); for a full-array sum the per-shard partials must add up
to the whole sum within the reductions' rtol 1e-5.  The BASELINE configs
must shard the way the scope table says (rows of C2 and C3, M of C5 with B
and bias whole, 2^31 / N elements of C4 plus a sum combine).
"""

from __future__ import annotations

import json

import numpy as np
import pytest

from conftest import CASES

from emmy_ptx_compiler_b200 import frontend, shard
from emmy_ptx_compiler_b200.errors import UnsupportedIR


def _load(cid: str):
    ir_path = next((CASES / cid).glob("*.ir.json"))
    raw = json.loads(ir_path.read_text())
    info = frontend.load_graph(raw)
    mk = frontend.load_meta_kernel(ir_path, info.kop.name)
    shapes, dtypes = frontend.load_shapes(raw, info.kop, mk)
    return raw, info.kop, mk, shapes, dtypes


def _oracle_kop(raw: dict, kop):
    """The shard IR decoded by the oracle's own IR classes (through its repr text)."""
    from emmy._core import Graph, KernelOp
    raw = json.loads(json.dumps(raw))
    for nd in raw["nodes"].values():
        if nd["op"] == "KernelOp":
            nd["op_fields"]["body"] = [repr(kop.body[0])]
    g = Graph.from_dict(raw)
    return next(n.op for n in g.nodes.values() if isinstance(n.op, KernelOp))


@pytest.mark.parametrize("cid,axis,cut", [
    ("c2_gelu_full", "a0", ["x", "y"]),
    ("c3_rowsummax_full", "a0", ["max_1", "sum_1", "x"]),
    ("c5_gemm_full", "i", ["A", "C"]),
])
def test_baseline_row_configs_shard_by_rows(cid, axis, cut):
    raw, kop, mk, shapes, dtypes = _load(cid)
    for parts in (1, 2, 8):
        spans = []
        for part in range(parts):
            sh = shard.shard_kernel(kop, shapes, parts, part)
            assert sh.mode == "rows" and sh.axis == axis and sh.buffers == cut
            for b in cut:
                assert sh.shapes[b] == (sh.hi - sh.lo,) + tuple(shapes[b])[1:]
            for b in set(shapes) - set(cut):
                assert sh.shapes[b] == shapes[b]
            spans.append((sh.lo, sh.hi))
        assert spans[0][0] == 0 and spans[-1][1] == sh.extent
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))


def test_full_sum_shards_into_partials():
    raw, kop, mk, shapes, dtypes = _load("c4_sum_full")
    sh = shard.shard_kernel(kop, shapes, 8, 3)
    assert sh.mode == "partial" and sh.combine == "add" and sh.buffers == ["x"]
    assert sh.shapes["x"] == ((1 << 31) // 8,)
    assert (sh.lo, sh.hi) == (3 << 28, 4 << 28)


@pytest.mark.parametrize("cid", ["c2_gelu_64x1000", "c3_rowsummax_64x5000", "m_matmul_f32_bias_96x160x80",
                                 "f_softmax_64x1000", "p_add2d_32x64"])
@pytest.mark.parametrize("parts", [2, 3])
def test_row_shards_concatenate_to_the_whole(cid, parts):
    import interp
    raw, kop, mk, shapes, dtypes = _load(cid)
    okop, meta, omk, oshapes, odtypes = interp.load_case(CASES / cid)
    inputs = interp.make_inputs(omk, oshapes, odtypes)
    outs = {a["name"]: tuple(a["shape"]) for a in omk["args"] if a.get("output")}
    whole = interp.evaluate(okop, oshapes, odtypes, inputs, outs)
    pieces = {n: [] for n in outs}
    for part in range(parts):
        sh = shard.shard_kernel(kop, shapes, parts, part)
        assert sh.mode == "rows"
        skop = _oracle_kop(raw, sh.kop)
        sin = {n: (v[sh.lo:sh.hi] if n in sh.buffers else v) for n, v in inputs.items()}
        souts = {n: sh.shapes[n] for n in outs}
        got = interp.evaluate(skop, {**oshapes, **{b: sh.shapes[b] for b in sh.buffers}}, odtypes, sin, souts)
        for n in outs:
            pieces[n].append(got[n])
    for n in outs:
        cat = np.concatenate(pieces[n], axis=0)
        assert np.array_equal(cat.view(np.uint32), whole[n].view(np.uint32)), n


def test_partial_sums_add_up_to_the_whole():
    import interp
    raw, kop, mk, shapes, dtypes = _load("c4_sum_1048579")
    okop, meta, omk, oshapes, odtypes = interp.load_case(CASES / "c4_sum_1048579")
    inputs = interp.make_inputs(omk, oshapes, odtypes)
    whole = float(interp.evaluate(okop, oshapes, odtypes, inputs, {"sum_1": ()})["sum_1"].reshape(-1)[0])
    total = 0.0
    for part in range(4):
        sh = shard.shard_kernel(kop, shapes, 4, part)
        skop = _oracle_kop(raw, sh.kop)
        got = interp.evaluate(skop, {**oshapes, "x": sh.shapes["x"]}, odtypes,
                              {"x": inputs["x"][sh.lo:sh.hi]}, {"sum_1": ()})
        total += float(got["sum_1"].reshape(-1)[0])
    exact = float(inputs["x"].astype(np.float64).sum())
    assert abs(total - whole) <= 1e-5 * abs(exact) + 1e-4
    assert abs(total - exact) <= 1e-5 * abs(exact) + 1e-4


def test_split_is_contiguous_and_even():
    assert [shard.split(10, 3, p) for p in range(3)] == [(0, 3), (3, 6), (6, 10)]
    with pytest.raises(ValueError):
        shard.split(10, 3, 3)


def test_what_does_not_shard_is_refused():
    raw, kop, mk, shapes, dtypes = _load("r_atomic_sum_512")
    with pytest.raises(UnsupportedIR):
        shard.shard_kernel(kop, shapes, 2, 0)
    raw, kop, mk, shapes, dtypes = _load("c4_sum_1")
    with pytest.raises(UnsupportedIR):
        shard.shard_kernel(kop, shapes, 2, 0)       # one element cannot be split in two
