"""The CPU oracle against independent expectations and against golden vectors
captured from the reference's own PTX on a B200 (CPU only)."""

from __future__ import annotations

import json
import math

import numpy as np
import pytest

from conftest import CASES, GOLDEN, small_cases


def _run(cid):
    import interp
    return interp.run_case(CASES / cid)


def test_add_is_exact():
    out, ins = _run("c1_add_64")
    assert np.array_equal(out["c"], ins["a"] + ins["b"])


def test_gelu_matches_float64_formula():
    out, ins = _run("c2_gelu_64x1000")
    z = ins["x"].astype(np.float64) * ins["s"] + ins["t"]
    ref = 0.5 * z * (1.0 + np.tanh(math.sqrt(2 / math.pi) * (z + 0.044715 * z ** 3)))
    np.testing.assert_allclose(out["y"], ref, rtol=2e-5, atol=2e-6)


def test_row_sum_max_against_float64():
    out, ins = _run("c3_rowsummax_64x5000")
    x = ins["x"].astype(np.float64)
    np.testing.assert_allclose(out["sum_1"], x.sum(-1), rtol=1e-5, atol=1e-4)
    assert np.array_equal(out["max_1"], ins["x"].max(-1))


def test_full_sum_and_mean_against_float64():
    out, ins = _run("c4_sum_1048579")
    assert abs(out["sum_1"][0] - ins["x"].astype(np.float64).sum()) < 1e-2
    out, ins = _run("r_mean_777")
    assert abs(out["mean"][0] - ins["x"].astype(np.float64).mean()) < 1e-6


def test_bf16_gemm_against_float64():
    import interp
    out, ins = _run("c5_gemm_256x512x512")
    acc = ins["A"].astype(np.float64) @ ins["B"].astype(np.float64) + ins["bias"]
    ref = interp.bf16_round(np.maximum(acc, 0).astype(np.float32))
    np.testing.assert_allclose(out["C"], ref, rtol=1e-2, atol=1e-2)


def test_strided_schedule_order_matches_a_plain_loop_restatement():
    """ora_strided_reduce_f32 against a direct Python restatement of the
    StridedLoop -> WarpShuffle -> TreeHalve order (compile.py:1866-1914, 2213-2286)."""
    import interp
    rng = np.random.default_rng(3)
    cols, bt = 777, 128
    x = rng.standard_normal((2, cols)).astype(np.float32)
    out = np.empty(2, np.float32)
    lib = interp.lib()
    lib.ora_strided_reduce_f32(interp._p(x), None, 2, cols, bt, 0, np.float32(0), interp._p(out))
    for r in range(2):
        acc = [np.float32(0)] * bt
        for t in range(bt):
            for k in range(t, cols, bt):
                acc[t] = np.float32(acc[t] + x[r, k])
        for s in (16, 8, 4, 2, 1):
            acc = [np.float32(acc[t] + acc[(t & ~31) | ((t & 31) ^ s)]) for t in range(bt)]
        sm = [acc[w * 32] for w in range(bt // 32)]
        step = len(sm) // 2
        while step:
            for w in range(step):
                sm[w] = np.float32(sm[w] + sm[w + step])
            step //= 2
        assert out[r] == sm[0]


def test_naive_gemm_is_sequential_fma():
    import interp
    rng = np.random.default_rng(5)
    A = rng.standard_normal((3, 9)).astype(np.float32)
    B = rng.standard_normal((9, 4)).astype(np.float32)
    C = np.empty((3, 4), np.float32)
    interp.lib().ora_gemm_seqfma_f32(interp._p(A), interp._p(B), interp._p(C), 3, 4, 9, 0)
    for i in range(3):
        for j in range(4):
            acc = np.float32(0)
            for k in range(9):
                acc = np.float32(np.float64(A[i, k]) * np.float64(B[k, j]) + np.float64(acc))
            assert abs(C[i, j] - acc) <= 2 * np.spacing(abs(acc))


GOLDEN_DIR = GOLDEN / "ref_outputs"


def _golden_ids():
    if not (GOLDEN_DIR / "INDEX.json").is_file():
        return []
    return sorted(json.loads((GOLDEN_DIR / "INDEX.json").read_text())["cases"])


@pytest.mark.parametrize("cid", _golden_ids() or ["<none captured>"])
def test_oracle_against_reference_ptx_golden_vectors(cid):
    """Golden vectors: outputs of the reference compiler's PTX run on a B200
    (tests/golden/capture_ref_outputs.py).  The oracle must reproduce them
    bit for bit where the reference arithmetic is IEEE-exact, and within the
    case's ulp bound where it uses the approximate ex2/lg2/rsqrt."""
    if cid == "<none captured>":
        pytest.skip("no golden vectors captured yet")
    import interp
    idx = json.loads((GOLDEN_DIR / "INDEX.json").read_text())["cases"][cid]
    data = np.load(GOLDEN_DIR / f"{cid}.npz")
    case_dir = CASES / idx["case_dir"]
    _, inputs = interp.run_case(CASES / cid)  # the parent case's inputs (bf16-rounded for GEMMs)
    out, _ = interp.run_case(case_dir, inputs)
    meta = json.loads((CASES / cid / "meta.json").read_text())
    check = meta.get("check", {})
    for name in idx["outputs"]:
        ref = data[name].reshape(-1)
        got = out[name].reshape(-1)[: ref.size]
        if idx.get("approx"):
            ok, why = interp.within(got, ref, check.get("oracle", {"rtol": 4e-6, "atol": 2e-6}))
            assert ok, f"{cid}.{name}: {why}"
        elif "atomic" in cid:
            np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-5)
        else:
            assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), f"{cid}.{name}"


def _attn_scale(kop) -> float:
    """The score scale of the naive attention IR: its first ``Let`` of a literal."""
    stack = list(kop.body)
    while stack:
        s = stack.pop(0)
        val = getattr(s, "value", None)
        if type(s).__name__ == "Let" and hasattr(val, "value"):
            return float(np.float32(val.value))
        for attr in ("body",):
            stack = list(getattr(s, attr, ()) or ()) + stack
    raise AssertionError("no scale literal in the attention IR")


@pytest.mark.parametrize("cid", ["a_attn_64x32", "a_attn_100x48", "a_attn_256x64", "a_attn_krows_80x40"])
def test_attention_c_restatement(cid):
    """``ora_attn_naive_f32`` (the C restatement used for the bench's CPU arm)
    gives the Python oracle's values bit for bit, and matches the golden
    vectors of the reference's PTX run on a B200 within the oracle bound."""
    import interp
    kop, meta, mk, shapes, dtypes = interp.load_case(CASES / cid)
    out, inputs = interp.run_case(CASES / cid)
    q = np.ascontiguousarray(inputs["q"], dtype=np.float32)
    kname = "kt" if "kt" in inputs else next(n for n in inputs if n not in ("q", "v"))
    kmat = np.ascontiguousarray(inputs[kname], dtype=np.float32)
    v = np.ascontiguousarray(inputs["v"], dtype=np.float32)
    sq, d = q.shape
    sk, dv = v.shape
    if kmat.shape == (sk, d):
        kmat = np.ascontiguousarray(kmat.T)    # the restatement takes keys as [d, sk]
    got = np.empty((sq, dv), dtype=np.float32)
    rc = interp.lib().ora_attn_naive_f32(interp._p(q), interp._p(kmat), interp._p(v), interp._p(got),
                                         sq, sk, d, dv, _attn_scale(kop))
    assert rc == 0
    oname = next(iter(out))
    assert np.array_equal(got.reshape(-1).view(np.uint32), out[oname].reshape(-1).view(np.uint32))
    if (GOLDEN_DIR / f"{cid}.npz").is_file():
        ref = np.load(GOLDEN_DIR / f"{cid}.npz")[oname].reshape(-1)
        ok, why = interp.within(got.reshape(-1), ref, {"rtol": 4e-6, "atol": 2e-6})
        assert ok, why


@pytest.mark.parametrize("cid", ["s_cpasync_matmul_64x48x80", "s_cpasync16_matmul_32x64x48",
                                 "s_smem_matmul_48x32x64"])
def test_simt_oracle_on_cp_async_matmul_equals_sequential_fma(cid):
    """The oracle's lockstep SIMT evaluation of a cp.async-staged matmul
    schedule gives the sequential-fma GEMM (ora_gemm_seqfma_f32) bit for bit:
    the staging changes where operands come from, not the order of the k sum."""
    import interp
    out, ins = interp.run_case(CASES / cid)
    A = np.ascontiguousarray(ins["A"], np.float32)
    B = np.ascontiguousarray(ins["B"], np.float32)
    C = np.empty(out["C"].shape, np.float32)
    interp.lib().ora_gemm_seqfma_f32(interp._p(A), interp._p(B), interp._p(C), A.shape[0], B.shape[1], A.shape[1], 0)
    assert np.array_equal(C.view(np.uint32), out["C"].view(np.uint32))


def _block_cooperative_cases():
    out = []
    for c in json.loads((CASES / "INDEX.json").read_text())["cases"]:
        cid = c["id"]
        if "_full" in cid or "2p28" in cid or "_prof_" in cid or "_bench_" in cid:
            continue
        text = next((CASES / cid).glob("*.ir.json")).read_text()
        if "TreeHalve" in text or "WarpShuffle" in text:
            out.append(cid)
    return out


@pytest.mark.parametrize("cid", _block_cooperative_cases())
def test_lockstep_simt_evaluation_agrees_with_the_schedule_evaluators(cid):
    """Two independent restatements of the reference's block-cooperative
    semantics: the oracle's schedule-specific evaluators (strided accumulate,
    butterfly, smem tree, in the reference's order) and its lockstep SIMT
    evaluation of the same IR, thread block by thread block.  Bit-identical."""
    import interp
    kop, meta, mk, shapes, dtypes = interp.load_case(CASES / cid)
    out, ins = interp.run_case(CASES / cid)
    outs = {a["name"]: tuple(a["shape"]) for a in mk["args"] if a.get("output")}
    simt = interp._eval_simt(kop, shapes, dtypes, ins, outs, {"grid": mk.get("grid"), "block": mk.get("block")})
    for name in out:
        assert np.array_equal(np.asarray(out[name]).view(np.uint32), np.asarray(simt[name]).view(np.uint32)), name
