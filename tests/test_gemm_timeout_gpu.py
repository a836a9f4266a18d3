"""Failure detection in the tcgen05 GEMM without a GPU fault: every mbarrier
wait is bounded, and a wait that runs out raises an EMMY_STATUS_TIMEOUT_* bit,
lets the CTA pair drain its in-flight loads and MMAs, frees its tensor
memory and returns.

A test-only build of the CTA-pair kernel leaves out one CTA's first TMA load
(cluster 0, first tile), so that the leader's pipeline stage never fills,
with every wait limited to 5 ms.  The launch must end by itself with a
timeout bit in the module's status word; the context must stay usable and
the next launch of the normal kernel - which allocates all 512 tensor-memory
columns of every SM it runs on, so it could not start if the aborted CTAs had
kept theirs - must match the oracle.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import CASES

pytestmark = pytest.mark.gpu

TIMEOUTS = 0x1 | 0x2 | 0x4   # EMMY_STATUS_TIMEOUT_PRODUCER | _MMA | _EPILOGUE


def test_gemm_wait_runs_out_and_the_next_launch_is_correct(cuda_device):
    import time

    import interp
    import torch
    from emmy_ptx_compiler_b200 import harness

    cid = "c5_gemm_256x512x512"
    faulty = harness.DeviceCase(CASES / cid, cuda_device,
                                options={"gemm_tune": {"skip_first_load": True, "wait_ns": 5_000_000}})
    assert faulty.bundle["notes"]["kernel"] == "tcgen05_pair"
    want, inputs = interp.run_case(CASES / cid)
    bufs = faulty.buffers(inputs)
    t0 = time.perf_counter()
    faulty.launch(bufs)
    torch.cuda.synchronize(cuda_device)
    elapsed = time.perf_counter() - t0
    st = faulty.module.status()
    assert st & TIMEOUTS, f"status 0x{st:x}"
    assert elapsed < 5.0, elapsed
    faulty.module.close()
    for _ in range(2):
        normal = harness.DeviceCase(CASES / cid, cuda_device)
        got = normal.run(inputs)          # raises on a non-zero status
        np.testing.assert_allclose(got["C"].reshape(-1), want["C"].reshape(-1), rtol=1e-2, atol=1e-2)
        normal.module.close()
