"""Attention family launch paths (no reference counterpart).

Two kernels lower the naive attention IR: the tensor-core kernel
(families/attention_tc.py, tcgen05 kind::tf32 with a three-term split, the
default) and the exact CUDA-core kernel (``attention_kernel: "exact"``, every
score and weighted sum in the reference's sequential fma order).

* Both read operands with 16-byte loads when the base pointers are 16-byte
  aligned, and with 4-byte loads otherwise; both paths must give the same
  bytes.
* The tensor-core kernel must stay within the attention bar (rtol 1e-4,
  atol 1e-5) of the exact kernel and of the CPU oracle, on every fixture and
  at the bench shape, and repeat its bits from launch to launch.
"""

from __future__ import annotations

import pytest

from conftest import CASES

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kernel", ["exact", "tc"])
@pytest.mark.parametrize("cid", ["a_attn_64x32", "a_attn_256x64", "a_attn_100x48"])
def test_unaligned_kv_matches_aligned(cid, kernel, cuda_device):
    import torch
    from emmy_ptx_compiler_b200 import harness
    case = harness.DeviceCase(CASES / cid, cuda_device, options={"attention_kernel": kernel})
    bufs = harness._seeded_device_inputs(case.spec, cuda_device, seed=5)
    case.launch(bufs)
    torch.cuda.synchronize(cuda_device)
    out_name = case.spec.outputs[0]
    aligned = bufs[out_name].clone()
    moved = dict(bufs)
    for name in case.spec.arg_order:
        if name in case.spec.outputs or name == case.spec.arg_order[0]:
            continue
        t = bufs[name]
        store = torch.empty(t.numel() + 1, dtype=t.dtype, device=t.device)
        view = store[1:].view(t.shape)      # 4 bytes past a 256-byte boundary
        view.copy_(t)
        assert view.data_ptr() % 16 == 4
        moved[name] = view
    moved[out_name] = torch.full_like(aligned, float("nan"))
    case.launch(moved)
    torch.cuda.synchronize(cuda_device)
    assert case.module.status() == 0
    assert torch.equal(moved[out_name].view(torch.int32), aligned.view(torch.int32))
    case.module.close()


def test_register_tiled_first_pass_matches_tiled_pass(cuda_device):
    """At the bench shape (2048 keys) the first pass runs as a register tile
    (every thread: all rows x four keys, k straight from L2).  Its output must
    be the tiled pass's bit for bit (each score is still one fma chain in d
    order), and both match the C restatement of the IR within the oracle bound."""
    import sys
    import numpy as np
    import torch
    from emmy_ptx_compiler_b200 import harness
    from conftest import REPO
    sys.path.insert(0, str(REPO / "oracle"))
    import interp
    cid = "a_attn_bench_2048x64"
    fast = harness.DeviceCase(CASES / cid, cuda_device, options={"attention_kernel": "exact"})
    tiled = harness.DeviceCase(CASES / cid, cuda_device,
                               options={"attention_kernel": "exact", "attention_first_pass": "tiled"})
    assert fast.bundle["notes"]["register_tiled_first_pass"] and not tiled.bundle["notes"]["register_tiled_first_pass"]
    bufs = harness._seeded_device_inputs(fast.spec, cuda_device, seed=9)
    outs = {}
    for name, case in (("fast", fast), ("tiled", tiled)):
        b = dict(bufs)
        b["attn"] = torch.full_like(bufs["attn"], float("nan"))
        case.launch(b)
        torch.cuda.synchronize(cuda_device)
        assert case.module.status() == 0
        outs[name] = b["attn"].cpu().numpy()
        case.module.close()
    assert np.array_equal(outs["fast"].view(np.uint32), outs["tiled"].view(np.uint32))
    q, kt, v = (bufs[n].cpu().numpy() for n in ("q", "kt", "v"))
    rows = 96                      # the C restatement on the first rows
    ref = np.empty((rows, 64), np.float32)
    assert interp.lib().ora_attn_naive_f32(interp._p(np.ascontiguousarray(q[:rows])), interp._p(kt), interp._p(v),
                                           interp._p(ref), rows, 2048, 64, 64, float(np.float32(1 / 8))) == 0
    ok, why = interp.within(outs["fast"][:rows], ref, {"rtol": 4e-6, "atol": 2e-6})
    assert ok, why


@pytest.mark.parametrize("exchange", ["grid", "cluster"])
@pytest.mark.parametrize("cid", ["a_attn_64x32", "a_attn_256x64", "a_attn_100x48", "a_attn_krows_80x40",
                                 "a_attn_bench_2048x64"])
def test_tensor_core_kernel_matches_the_exact_kernel(cid, exchange, cuda_device):
    import torch
    from emmy_ptx_compiler_b200 import harness
    tc = harness.DeviceCase(CASES / cid, cuda_device, options={"attention_kernel": "tc", "attention_exchange": exchange})
    ex = harness.DeviceCase(CASES / cid, cuda_device, options={"attention_kernel": "exact"})
    assert tc.bundle["notes"]["kernel"] == "attention_tcgen05_tf32x3"
    assert tc.bundle["notes"]["exchange"] == exchange
    bufs = harness._seeded_device_inputs(tc.spec, cuda_device, seed=13)
    out = tc.spec.outputs[0]
    got = {}
    for name, case in (("tc", tc), ("tc_again", tc), ("exact", ex)):
        b = dict(bufs)
        b[out] = torch.full_like(bufs[out], float("nan"))
        case.launch(b)
        torch.cuda.synchronize(cuda_device)
        assert case.module.status() == 0, name
        got[name] = b[out]
    assert torch.equal(got["tc"].view(torch.int32), got["tc_again"].view(torch.int32))
    err = (got["tc"] - got["exact"]).abs()
    bad = int((err > 1e-5 + 1e-4 * got["exact"].abs()).sum())
    assert bad == 0, (cid, float(err.max()))
    tc.module.close()
    ex.module.close()


@pytest.mark.parametrize("cid", ["a_attn_256x64", "a_attn_bench_2048x64", "a_attn_krows_80x40"])
def test_grid_and_cluster_exchanges_give_the_same_bits(cid, cuda_device):
    """The CTAs of a query tile combine their row values and partial outputs
    in CTA order either way: through distributed shared memory (a cluster) or
    through global memory under a cooperative launch.  The bits must agree,
    launch after launch (the grid exchange's counters return to zero)."""
    import torch
    from emmy_ptx_compiler_b200 import harness
    cases = {x: harness.DeviceCase(CASES / cid, cuda_device, options={"attention_kernel": "tc", "attention_exchange": x})
             for x in ("grid", "cluster")}
    bufs = harness._seeded_device_inputs(cases["grid"].spec, cuda_device, seed=17)
    out = cases["grid"].spec.outputs[0]
    got = {}
    for name in ("grid", "cluster", "grid2", "grid3"):
        case = cases[name.rstrip("23")]
        b = dict(bufs)
        b[out] = torch.full_like(bufs[out], float("nan"))
        case.launch(b)
        torch.cuda.synchronize(cuda_device)
        assert case.module.status() == 0, name
        got[name] = b[out].view(torch.int32)
    for name in ("cluster", "grid2", "grid3"):
        assert torch.equal(got["grid"], got[name]), name
    for case in cases.values():
        case.module.close()


def test_grid_exchange_rejects_a_grid_beyond_its_exchange_slots(cuda_device):
    """A launch with more CTAs than the module's exchange slots raises
    EMMY_STATUS_BAD_LAUNCH before any CTA waits on another, and the next
    launch under the launch record is correct."""
    import torch
    from emmy_ptx_compiler_b200 import harness
    case = harness.DeviceCase(CASES / "a_attn_256x64", cuda_device, options={"attention_exchange": "grid"})
    assert case.bundle["notes"]["exchange"] == "grid"
    g = case.bundle["launch"]["grid"][0]
    bufs = harness._seeded_device_inputs(case.spec, cuda_device, seed=3)
    out = case.spec.outputs[0]
    case.launch(bufs)
    torch.cuda.synchronize(cuda_device)
    want = bufs[out].clone()
    bufs[out].fill_(float("nan"))
    case.launch(bufs, grid=[g + case.bundle["notes"]["ctas_per_tile"], 1, 1], block=[512, 1, 1])
    torch.cuda.synchronize(cuda_device)
    assert case.module.status() == 0x8       # EMMY_STATUS_BAD_LAUNCH
    assert bool(torch.isnan(bufs[out]).all())
    case.launch(bufs)
    torch.cuda.synchronize(cuda_device)
    assert case.module.status() == 0
    assert torch.equal(bufs[out].view(torch.int32), want.view(torch.int32))
    case.module.close()


def test_grid_exchange_range_launches_compose(cuda_device):
    """Launches over the two query tiles separately give the whole launch's
    bits; the CTAs of the tile outside a range wait for nothing."""
    import torch
    from emmy_ptx_compiler_b200 import harness
    case = harness.DeviceCase(CASES / "a_attn_256x64", cuda_device, options={"attention_exchange": "grid"})
    assert case.bundle["notes"]["exchange"] == "grid"
    bufs = harness._seeded_device_inputs(case.spec, cuda_device, seed=23)
    out = case.spec.outputs[0]
    case.launch(bufs)
    torch.cuda.synchronize(cuda_device)
    whole = bufs[out].clone()
    bufs[out].fill_(float("nan"))
    order = [bufs[n] for n in case.spec.arg_order]
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    case.module.launch_range(order, 128, 256, stream=stream)
    torch.cuda.synchronize(cuda_device)
    assert bool(torch.isnan(bufs[out][:128]).all())
    case.module.launch_range(order, 0, 128, stream=stream)
    torch.cuda.synchronize(cuda_device)
    assert case.module.status() == 0
    assert torch.equal(bufs[out].view(torch.int32), whole.view(torch.int32))
    case.module.close()


def test_grid_exchange_wait_runs_out_and_the_next_launch_is_correct(cuda_device):
    """Failure detection of the grid exchange without a GPU fault: a test-only
    build in which CTA 1 leaves out its first arrival at its tile's barrier,
    with every wait limited to 5 ms.  The other CTAs of the tile wait out
    their limit, the launch ends by itself with EMMY_STATUS_TIMEOUT_REDUCE,
    and a freshly loaded normal module (its barrier counters start at zero)
    gives the cluster exchange's bits."""
    import time

    import torch
    from emmy_ptx_compiler_b200 import harness
    cid = "a_attn_bench_2048x64"
    faulty = harness.DeviceCase(CASES / cid, cuda_device,
                                options={"attention_exchange": "grid",
                                         "attention_tune": {"skip_first_arrive": True, "wait_ns": 5_000_000}})
    assert faulty.bundle["notes"]["exchange"] == "grid"
    bufs = harness._seeded_device_inputs(faulty.spec, cuda_device, seed=29)
    out = faulty.spec.outputs[0]
    t0 = time.perf_counter()
    faulty.launch(bufs)
    torch.cuda.synchronize(cuda_device)
    elapsed = time.perf_counter() - t0
    st = faulty.module.status()
    assert st & 0x20, f"status 0x{st:x}"          # EMMY_STATUS_TIMEOUT_REDUCE
    assert elapsed < 5.0, elapsed
    faulty.module.close()
    ref = harness.DeviceCase(CASES / cid, cuda_device, options={"attention_exchange": "cluster"})
    b = dict(bufs)
    b[out] = torch.full_like(bufs[out], float("nan"))
    ref.launch(b)
    torch.cuda.synchronize(cuda_device)
    assert ref.module.status() == 0
    want = b[out].clone()
    ref.module.close()
    for _ in range(2):
        normal = harness.DeviceCase(CASES / cid, cuda_device, options={"attention_exchange": "grid"})
        b[out].fill_(float("nan"))
        normal.launch(b)
        torch.cuda.synchronize(cuda_device)
        assert normal.module.status() == 0
        assert torch.equal(b[out].view(torch.int32), want.view(torch.int32))
        normal.module.close()
