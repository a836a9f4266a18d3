"""Full BASELINE-size configs on the GPU, checked through properties that do
not need a full CPU re-computation: sampled rows against the CPU oracle,
exact maxima, an f64 checksum of the 2^31-element sum, and bit-exact
reproducibility of repeated launches."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import CASES

pytestmark = pytest.mark.gpu


def _device_inputs(spec, seed: int = 0):
    import torch
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    bufs = {}
    for name in spec.arg_order:
        a = spec.args[name]
        shape = tuple(a["shape"]) or (1,)
        dt = {"f32": torch.float32, "bf16": torch.bfloat16}[a.get("dtype", "f32")]
        if a.get("output"):
            bufs[name] = torch.zeros(shape, dtype=dt, device="cuda")
            continue
        init = a["init"]
        t = torch.empty(shape, dtype=torch.float32, device="cuda")
        if init["kind"] == "uniform":
            t.uniform_(init["low"], init["high"], generator=g)
        else:
            t.normal_(init.get("mean", 0.0), init.get("std", 1.0), generator=g)
        bufs[name] = t.to(dt)
    return bufs


def _run(case, bufs):
    import torch
    case.launch(bufs)
    torch.cuda.synchronize()
    assert case.module.status() == 0


def test_c2_gelu_full(cuda_device):
    import interp
    from emmy_ptx_compiler_b200 import harness
    case = harness.DeviceCase(CASES / "c2_gelu_full", cuda_device)
    bufs = _device_inputs(case.spec)
    _run(case, bufs)
    y1 = bufs["y"].clone()
    _run(case, bufs)
    assert bool((y1 == bufs["y"]).all())
    rows = [0, 1, 8191, 16383]
    kop, meta, mk, shapes, dtypes = interp.load_case(CASES / "c2_gelu_64x1000")
    import copy
    from emmy._core import Axis, Dim
    tile = copy.copy(list(kop.body)[0])
    tile.axes = (Axis("a0", Dim(len(rows))), Axis("a1", Dim(16384)))
    kop = copy.copy(kop)
    kop.body = (tile,)
    x = bufs["x"][rows].float().cpu().numpy()
    s, t = bufs["s"].cpu().numpy(), bufs["t"].cpu().numpy()
    want = interp.evaluate(kop, {"x": x.shape, "s": (16384,), "t": (16384,), "y": x.shape},
                           dtypes, {"x": x, "s": s, "t": t}, {"y": x.shape})["y"]
    got = bufs["y"][rows].cpu().numpy()
    ok, why = interp.within(got, want, meta["check"]["oracle"])
    assert ok, why
    case.module.close()


def test_c3_rowsummax_full(cuda_device):
    import interp
    from emmy_ptx_compiler_b200 import harness
    case = harness.DeviceCase(CASES / "c3_rowsummax_full", cuda_device)
    bufs = _device_inputs(case.spec)
    _run(case, bufs)
    s1, m1 = bufs["sum_1"].clone(), bufs["max_1"].clone()
    _run(case, bufs)
    assert bool((s1 == bufs["sum_1"]).all()) and bool((m1 == bufs["max_1"]).all())
    import torch
    assert bool((bufs["max_1"] == bufs["x"].max(dim=1).values).all())
    rows = [0, 4095, 8191]
    x = bufs["x"][rows].cpu().numpy()
    ref = np.empty(len(rows), np.float64)
    interp.lib().ora_row_sum_f64(interp._p(np.ascontiguousarray(x)), len(rows), x.shape[1], interp._p(ref))
    np.testing.assert_allclose(bufs["sum_1"][rows].cpu().numpy(), ref, rtol=1e-5, atol=1e-3)
    del torch
    case.module.close()


def test_c4_sum_full(cuda_device):
    import torch
    from emmy_ptx_compiler_b200 import harness
    case = harness.DeviceCase(CASES / "c4_sum_full", cuda_device)
    bufs = _device_inputs(case.spec)
    _run(case, bufs)
    a = float(bufs["sum_1"].item())
    _run(case, bufs)
    assert float(bufs["sum_1"].item()) == a, "the chunked combine is deterministic"
    # f64 checksum on the host, 256 MiB at a time
    x = bufs["x"]
    total = 0.0
    step = 1 << 26
    for i in range(0, x.numel(), step):
        total += float(x[i:i + step].cpu().numpy().astype(np.float64).sum())
    assert abs(a - total) <= 1e-5 * max(1.0, abs(total)) + 0.05, (a, total)
    del torch
    case.module.close()


def test_c5_gemm_full(cuda_device):
    import interp
    import torch
    from emmy_ptx_compiler_b200 import harness
    case = harness.DeviceCase(CASES / "c5_gemm_full", cuda_device)
    assert case.bundle["notes"]["kernel"] in ("tcgen05", "tcgen05_pair")
    bufs = _device_inputs(case.spec)
    _run(case, bufs)
    c1 = bufs["C"].clone()
    _run(case, bufs)
    assert bool((c1 == bufs["C"]).all())
    rows = [0, 127, 128, 5000, 16383]
    A = bufs["A"][rows].float().cpu().numpy()
    B = bufs["B"].float().cpu().numpy()
    bias = bufs["bias"].cpu().numpy()
    acc = np.empty((len(rows), B.shape[1]), np.float32)
    interp.lib().ora_gemm_seqfma_f32(interp._p(np.ascontiguousarray(A)), interp._p(np.ascontiguousarray(B)),
                                     interp._p(acc), len(rows), B.shape[1], B.shape[0], 0)
    want = interp.bf16_round(np.maximum(acc + bias, 0).astype(np.float32))
    got = bufs["C"][rows].float().cpu().numpy()
    np.testing.assert_allclose(got, want, rtol=1e-2, atol=1e-2)
    del torch
    case.module.close()
