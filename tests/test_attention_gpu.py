"""Attention family launch paths (no reference counterpart).

Key and value tiles are copied into shared memory with 16-byte asynchronous
copies when the base pointers are 16-byte aligned, and with plain loads
otherwise (every chunk address is the base plus a multiple of 16 bytes, so
the base decides).  Both paths must give the same bytes.
"""

from __future__ import annotations

import pytest

from conftest import CASES

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cid", ["a_attn_64x32", "a_attn_256x64", "a_attn_100x48"])
def test_unaligned_kv_matches_aligned(cid, cuda_device):
    import torch
    from emmy_ptx_compiler_b200 import harness
    case = harness.DeviceCase(CASES / cid, cuda_device)
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
