"""The schedule family (any KernelOp, lowered in the schedule its IR spells
out) against the reference compiler's PTX on the same GPU.

Every small fixture is compiled a second time with ``family="schedule"``,
the lowering used for IRs no other family recognises.  It runs under
the meta.json launch, as the reference's PTX does.  Because it issues the
reference's instructions in the reference's order, its outputs must equal the
reference PTX's bit for bit.  There are three exceptions:

- atomic accumulations, whose order the hardware picks;
- the attention IRs, where the reference rewrites single-warp loops into a
  different summation order;
- bf16 GEMMs, which the reference can only run on f32 copies; the host
  rounds that output to bf16, which our bf16 store does as well.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import CASES, small_cases
from test_parity_gpu import _ref_dir, _run_reference

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cid", small_cases())
def test_schedule_family_matches_reference_ptx(cid, cuda_device):
    import interp
    from emmy_ptx_compiler_b200 import harness

    ref_dir = _ref_dir(cid)
    if ref_dir is None:
        pytest.skip("no reference PTX for this IR")
    case = harness.DeviceCase(CASES / cid, cuda_device, options={"family": "schedule"})
    assert case.bundle["family"] == "schedule"
    _, inputs = interp.run_case(CASES / cid)
    ours = case.run(inputs)
    ref = _run_reference(ref_dir, inputs, cuda_device)
    check = case.spec.meta.get("check", {})
    for name in case.spec.outputs:
        o = ours[name].reshape(-1)
        r = ref[name].reshape(-1)
        if ref_dir.name == "ref_f32":
            r = interp.bf16_round(r)
        if "atomic" in cid or cid.startswith("a_attn"):
            np.testing.assert_allclose(o, r, rtol=check.get("rtol", 1e-5), atol=check.get("atol", 1e-5),
                                       err_msg=f"{cid}.{name}")
        else:
            assert np.array_equal(o.view(np.uint32), r.view(np.uint32)), \
                f"{cid}.{name}: {int((o.view(np.uint32) != r.view(np.uint32)).sum())} elements differ"
    case.module.close()
