"""Unit-range launches and the chunk-pipelined host path (no reference
counterpart: the reference runner launched whole problems only).

* A module launched over consecutive unit ranges (pointwise: cells, GEMM:
  output rows) produces exactly the bytes of one whole launch, and a range
  launch writes nothing outside its range.
* ``emmy_run_host`` on a problem large enough to be pipelined (copy-in,
  kernel and copy-out of successive chunks on three streams) returns exactly
  the outputs of a device launch.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import CASES

pytestmark = pytest.mark.gpu


def _device_inputs(case, device):
    from emmy_ptx_compiler_b200 import harness
    return harness._seeded_device_inputs(case.spec, device, seed=7)


def _ranges(total: int, align: int, pieces: list[int]) -> list[tuple[int, int]]:
    """Consecutive ranges of ``pieces`` alignment units each, the last one ending at ``total``."""
    out, b = [], 0
    for p in pieces:
        e = min(total, b + p * align)
        if b < e:
            out.append((b, e))
        b = e
    if b < total:
        out.append((b, total))
    return out


@pytest.mark.parametrize("cid,pieces", [
    ("c2_gelu_64x1000", [1, 3, 2]),
    ("p_add2d_32x64", [0]),
    ("c5_gemm_520x320x392", [1, 1]),      # CTA-pair tiles of 256 rows, last range 8 rows
    ("c5_gemm_384x1024x768", [1]),
    ("c5_gemm_128x64x256", [1]),
    ("c5_gemm_200x136x300", [1, 2]),      # SIMT tiles of 64 rows
    ("f_softmax_64x1000", [3, 10]),       # row-fused: units are rows
    ("f_rmsnorm_7x4096", [2, 3]),         # row-fused, 16 KiB rows: one CTA per row of the range
    ("a_attn_100x48", [2, 5]),            # attention: blocks of 4 query rows
    ("a_attn_256x64", [1]),               # tensor-core attention, two query tiles
])
def test_ranges_compose_to_whole(cid, pieces, cuda_device):
    import torch
    from emmy_ptx_compiler_b200 import harness
    case = harness.DeviceCase(CASES / cid, cuda_device)
    total, align, per_unit = case.module.unit_range()
    assert total > 0 and align > 0
    bufs = _device_inputs(case, cuda_device)
    case.launch(bufs)
    torch.cuda.synchronize(cuda_device)
    whole = {n: bufs[n].clone() for n in case.spec.outputs}
    for n in case.spec.outputs:
        bufs[n].zero_()
    order = [bufs[n] for n in case.spec.arg_order]
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    rs = _ranges(total, align, pieces)
    for i, (b, e) in enumerate(rs):
        case.module.launch_range(order, b, e, stream=stream)
        torch.cuda.synchronize(cuda_device)
        if i == 0:
            # nothing outside the first range was written
            for k, n in enumerate(case.spec.arg_order):
                if n in case.spec.outputs and per_unit[k]:
                    flat = bufs[n].view(-1).view(torch.uint8)
                    assert int(flat[e * per_unit[k]:].count_nonzero()) == 0, f"{cid}: wrote past range"
    assert case.module.status() == 0
    for n in case.spec.outputs:
        assert torch.equal(bufs[n].view(torch.uint8), whole[n].view(torch.uint8)), \
            f"{cid}.{n}: {len(rs)} range launches differ from one whole launch"
    case.module.close()


def test_unaligned_range_is_rejected(cuda_device):
    from emmy_ptx_compiler_b200 import harness, runtime
    case = harness.DeviceCase(CASES / "c2_gelu_64x1000", cuda_device)
    total, align, _ = case.module.unit_range()
    bufs = _device_inputs(case, cuda_device)
    order = [bufs[n] for n in case.spec.arg_order]
    with pytest.raises(runtime.EmmyError):
        case.module.launch_range(order, 1, total)
    with pytest.raises(runtime.EmmyError):
        case.module.launch_range(order, 0, total + align)
    case.module.close()


@pytest.mark.parametrize("cid", ["c2_gelu_prof_4096x16384", "c5_gemm_prof_8192x8192x8192"])
def test_pipelined_host_path_matches_device_launch(cid, cuda_device):
    """Large enough to be chunked: 256 MiB in + 256 MiB out (pointwise), and
    A 128 MiB + C 128 MiB streamed with B read whole (GEMM)."""
    import torch
    from emmy_ptx_compiler_b200 import harness, runtime
    case = harness.DeviceCase(CASES / cid, cuda_device)
    bufs = _device_inputs(case, cuda_device)
    case.launch(bufs)
    torch.cuda.synchronize(cuda_device)
    host, ptrs, nbytes, roles = {}, [], [], []
    for n in case.spec.arg_order:
        t = bufs[n]
        h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
        if n in case.spec.outputs:
            h.fill_(7)  # overwritten by the call
            roles.append(runtime.EMMY_ROLE_OUT)
        else:
            h.copy_(t)
            roles.append(runtime.EMMY_ROLE_IN)
        host[n] = h
        ptrs.append(h.data_ptr())
        nbytes.append(h.numel() * h.element_size())
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    for _ in range(2):  # second call reuses the module's buffers, streams and events
        case.module.run_host(ptrs, nbytes, roles, stream=stream)
        for n in case.spec.outputs:
            assert torch.equal(host[n].view(torch.uint8), bufs[n].cpu().view(torch.uint8)), \
                f"{cid}.{n}: pipelined host path differs from the device launch"
    assert case.module.status() == 0
    case.module.close()


@pytest.mark.parametrize("cid,pinned", [
    ("c1_add_64", True),            # pointwise, 768 B: pinned host memory the kernel reads directly
    ("c1_add_64", False),           # same path from pageable buffers
    ("c2_gelu_3x7", True),
    ("f_softmax_33x130", True),     # row-fused, 34 KB
    ("c4_sum_1000", True),          # reduction: copy-engine path whatever the size
    ("c2_gelu_64x1000", False),     # 512 KB: above the small-payload bound
])
def test_small_host_path_matches_device_launch(cid, pinned, cuda_device):
    """``emmy_run_host`` on small problems returns exactly the outputs of a
    device launch, for every path it picks (and again on a second call)."""
    import torch
    from emmy_ptx_compiler_b200 import runtime
    from emmy_ptx_compiler_b200 import harness
    case = harness.DeviceCase(CASES / cid, cuda_device)
    bufs = _device_inputs(case, cuda_device)
    case.launch(bufs)
    torch.cuda.synchronize(cuda_device)
    zeroed = set(case.spec.meta.get("kernels", [{}])[0].get("zero_outputs", []))
    host, ptrs, nbytes, roles = {}, [], [], []
    for n in case.spec.arg_order:
        t = bufs[n]
        h = torch.empty(t.shape, dtype=t.dtype, pin_memory=pinned)
        if n in case.spec.outputs:
            h.fill_(7)
            roles.append(runtime.EMMY_ROLE_OUT_ZEROED if n in zeroed else runtime.EMMY_ROLE_OUT)
        else:
            h.copy_(t)
            roles.append(runtime.EMMY_ROLE_IN)
        host[n] = h
        ptrs.append(h.data_ptr())
        nbytes.append(h.numel() * h.element_size())
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    for _ in range(2):
        case.module.run_host(ptrs, nbytes, roles, stream=stream)
        for n in case.spec.outputs:
            assert torch.equal(host[n].view(torch.uint8), bufs[n].cpu().view(torch.uint8)), \
                f"{cid}.{n}: host path differs from the device launch"
    assert case.module.status() == 0
    case.module.close()


@pytest.mark.parametrize("cid", ["c2_gelu_256x4096", "c5_gemm_384x1024x768", "c5_gemm_520x320x392",
                                 "c5_gemm_bnk_384x256x512", "c5_gemm_200x136x300", "f_rmsnorm_7x4096",
                                 "a_attn_256x64"])
def test_sharded_launch_of_two_modules_on_one_device(cid, cuda_device):
    """emmy_launch_sharded over two modules loaded on the same GPU: the second
    shard's streamed buffers hold only its units, and the runtime rebases their
    pointers by the shard's first unit.  The GEMM's tensor map over A must then
    start at the shard's first row (it never points outside the buffer); the
    gathered result is bit-identical to one whole launch."""
    import torch
    from emmy_ptx_compiler_b200 import harness, runtime
    case = harness.DeviceCase(CASES / cid, cuda_device)
    bufs = harness._seeded_device_inputs(case.spec, cuda_device, seed=3)
    case.launch(bufs)
    torch.cuda.synchronize(cuda_device)
    want = {n: bufs[n].clone() for n in case.spec.outputs}
    mods = [case.module, runtime.Module(case.bundle["cubin"], case.spec.entry, cuda_device)]
    total, align, per_unit = case.module.unit_range()
    args, outs = [], []
    assert runtime.shard_range(mods[1], 2, 1)[0] > 0, "the second shard starts past unit 0"
    for d in range(2):
        b, e = runtime.shard_range(mods[d], 2, d)   # a shard may be empty (units of 128 rows)
        row, shard_out = [], {}
        for k, n in enumerate(case.spec.arg_order):
            full = bufs[n] if n not in case.spec.outputs else torch.zeros_like(bufs[n])
            flat = full.reshape(-1)
            t = flat[b * (per_unit[k] // full.element_size()):e * (per_unit[k] // full.element_size())].clone() \
                if per_unit[k] else full.clone()
            if n in case.spec.outputs:
                shard_out[n] = t
            row.append(t)
        args.append(row)
        outs.append(shard_out)
    runtime.launch_sharded(mods, args)
    torch.cuda.synchronize(cuda_device)
    assert mods[0].status() == 0 and mods[1].status() == 0
    for n in case.spec.outputs:
        got = torch.cat([outs[d][n].reshape(-1) for d in range(2)])
        assert torch.equal(got.view(torch.uint8), want[n].reshape(-1).view(torch.uint8)), f"{cid}.{n}"
    mods[1].close()
    case.module.close()
