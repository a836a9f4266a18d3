"""emmy_sum_f32_noalloc: the full-array sum for callers that cannot allocate.

Some callers embed this library under rules that forbid device allocation in
the call path - a fixed memory budget, a pre-sized pool, or a runtime that
owns every allocation and hands the library only its input and output
buffers.  For them the library exports one reduction entry point whose
cross-block scratch is a fixed array compiled into the library instead of
memory allocated per call.  This test calls it through the C ABI and checks
it against the existing module path (the compiled full-sum KernelOp,
launched with emmy_launch) on the same device buffer, twice in a row, with
the reductions' tolerance (rtol 1e-5).  The file is named so that pytest
collects it last.
"""

from __future__ import annotations

import pytest

from conftest import CASES

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cid", ["c4_sum_1048579", "c4_sum_chunk_2p28", "c4_sum_1000"])
def test_noalloc_sum_matches_the_module_path(cid, cuda_device):
    import torch
    from emmy_ptx_compiler_b200 import harness, runtime

    case = harness.DeviceCase(CASES / cid, cuda_device)
    n = int(case.spec.args["x"]["shape"][0])
    g = torch.Generator(device="cuda")
    g.manual_seed(11)
    x = torch.empty(n, dtype=torch.float32, device="cuda").uniform_(-1.0, 1.0, generator=g)
    ref = torch.zeros(1, dtype=torch.float32, device="cuda")
    case.launch({"x": x, "sum_1": ref})
    outs = []
    for _ in range(2):
        out = torch.full((1,), float("nan"), dtype=torch.float32, device="cuda")
        runtime.sum_f32_noalloc(x, n, out, device=cuda_device,
                                stream=torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        outs.append(float(out.item()))
    want = float(ref.item())
    for got in outs:
        assert abs(got - want) <= 1e-5 * abs(want) + 1e-4, (got, want)
    assert outs[0] == outs[1], "the shared scratch is reused cleanly by the next call"
    case.module.close()


@pytest.mark.parametrize("n,offset", [(0, 0), (1, 0), (1, 1), (1000, 1), ((1 << 20) + 3, 0),
                                      ((1 << 20) + 3, 1), ((1 << 22) + 5, 3)])
def test_noalloc_sum_against_an_f64_sum(n, offset, cuda_device):
    """Tiny sizes (n = 0 writes 0, n = 1), and x starting 4 or 12 bytes past a
    16-byte boundary, which takes the kernel's scalar path instead of its
    float4 path; the expected value is an f64 sum on the host."""
    import numpy as np
    import torch
    from emmy_ptx_compiler_b200 import runtime

    g = torch.Generator(device="cuda")
    g.manual_seed(5 + n)
    base = torch.empty(n + 4, dtype=torch.float32, device="cuda").uniform_(-1.0, 1.0, generator=g)
    x = base[offset:offset + n]
    assert (x.data_ptr() % 16 == 0) == (offset == 0)
    want = float(x.cpu().numpy().astype(np.float64).sum())
    outs = []
    for _ in range(2):
        out = torch.full((1,), float("nan"), dtype=torch.float32, device="cuda")
        runtime.sum_f32_noalloc(x, n, out, device=cuda_device, stream=torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        outs.append(float(out.item()))
    for got in outs:
        assert abs(got - want) <= 1e-5 * abs(want) + 1e-4, (got, want)
    if n == 0:
        assert outs == [0.0, 0.0]
    if n == 1:
        assert outs[0] == float(x.item())
    assert outs[0] == outs[1]


def test_noalloc_rejects_sizes_beyond_its_scratch(cuda_device):
    import ctypes
    from emmy_ptx_compiler_b200 import runtime

    lib = runtime.lib()
    too_many = (1 << 36) + 1
    # rejected on the host before any launch, so the pointers are never touched
    rc = lib.emmy_sum_f32_noalloc(cuda_device, 16, too_many, 16, 0)
    assert rc == -3
    buf = ctypes.create_string_buffer(512)
    lib.emmy_last_error(buf, 512)
    assert b"exceeds the maximum" in buf.value
