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
