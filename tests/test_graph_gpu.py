"""CUDA graphs of launches and bound launchers (no reference counterpart: the
reference leaves launching to its caller).

* A graph recorded from ``emmy_launch`` calls runs nothing while it records,
  and its replay writes exactly the bytes of the eager launch, for every kernel
  family (cluster launches and tensor-map parameters included).
* Replay reads the buffers as they are at replay time (pointers are
  recorded, not contents).
* ``Module.bind`` launches exactly what ``Module.launch`` does.
"""

from __future__ import annotations

import pytest

from conftest import CASES

pytestmark = pytest.mark.gpu


def _case(cid, device):
    from emmy_ptx_compiler_b200 import harness
    case = harness.DeviceCase(CASES / cid, device)
    bufs = harness._seeded_device_inputs(case.spec, device, seed=11)
    return case, bufs


def _fill_outputs(case, bufs, value=float("nan")):
    for n in case.spec.outputs:
        bufs[n].fill_(value)


@pytest.mark.parametrize("cid", [
    "c1_add_64",
    "c2_gelu_64x1000",          # pointwise, occupancy-sized grid
    "c5_gemm_384x1024x768",     # tcgen05 CTA pairs: cluster launch, tensor maps
    "c5_gemm_128x64x256",       # single-CTA tcgen05
    "f_softmax_64x1000",        # row-fused
    "a_attn_100x48",            # attention
])
def test_graph_replay_matches_eager(cid, cuda_device):
    import torch
    from emmy_ptx_compiler_b200 import runtime
    case, bufs = _case(cid, cuda_device)
    order = [bufs[n] for n in case.spec.arg_order]
    case.launch(bufs)
    torch.cuda.synchronize(cuda_device)
    eager = {n: bufs[n].clone() for n in case.spec.outputs}

    _fill_outputs(case, bufs)
    s = torch.cuda.Stream(device=cuda_device)
    torch.cuda.synchronize(cuda_device)
    with runtime.Graph.record(cuda_device, s.cuda_stream) as g:
        case.module.launch(order, stream=s.cuda_stream)
    torch.cuda.synchronize(cuda_device)
    for n in case.spec.outputs:  # recording ran nothing
        assert torch.isnan(bufs[n].float()).all(), n
    for _ in range(2):
        g.launch(s.cuda_stream)
    torch.cuda.synchronize(cuda_device)
    assert case.module.status() == 0
    for n in case.spec.outputs:
        assert torch.equal(bufs[n].view(torch.uint8), eager[n].view(torch.uint8)), n
    g.close()
    case.module.close()


def test_graph_replay_reads_current_buffers(cuda_device):
    import torch
    from emmy_ptx_compiler_b200 import runtime
    case, bufs = _case("c1_add_64", cuda_device)
    order = [bufs[n] for n in case.spec.arg_order]
    s = torch.cuda.Stream(device=cuda_device)
    torch.cuda.synchronize(cuda_device)
    with runtime.Graph.record(cuda_device, s.cuda_stream) as g:
        for _ in range(100):
            case.module.launch(order, stream=s.cuda_stream)
    bufs["a"].add_(1.0)
    torch.cuda.synchronize(cuda_device)
    g.launch(s.cuda_stream)
    torch.cuda.synchronize(cuda_device)
    assert torch.equal(bufs["c"], bufs["a"] + bufs["b"])
    g.close()
    case.module.close()


def test_graph_rejects_default_stream(cuda_device):
    from emmy_ptx_compiler_b200 import runtime
    with pytest.raises(runtime.EmmyError):
        with runtime.Graph.record(cuda_device, 0):
            pass


@pytest.mark.parametrize("cid", ["c1_add_64", "c2_gelu_64x1000", "c5_gemm_384x1024x768"])
def test_bound_launch_matches_launch(cid, cuda_device):
    import torch
    case, bufs = _case(cid, cuda_device)
    case.launch(bufs)
    torch.cuda.synchronize(cuda_device)
    eager = {n: bufs[n].clone() for n in case.spec.outputs}
    _fill_outputs(case, bufs)
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    go = case.module.bind([bufs[n] for n in case.spec.arg_order], stream=stream)
    go()
    go()
    torch.cuda.synchronize(cuda_device)
    for n in case.spec.outputs:
        assert torch.equal(bufs[n].view(torch.uint8), eager[n].view(torch.uint8)), n
    case.module.close()
