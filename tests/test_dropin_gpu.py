"""The CLI's PTX under the reference's launch contract, run by a runner that
is not this library.

``python compile.py kernel.ir.json > out.ptx`` must print a module a
reference-style runner can use unchanged (compile.py:854-864,
README.md:170-182): load the PTX, resolve ``.entry <KernelOp.name>``, pass
only the ``arg_order`` buffers (and scalars), and launch with meta.json's
grid, block and ``smem_bytes``.  This test is that runner, written against
the CUDA driver API through cuda-python (not libemmy_b200): for every small
fixture it compiles the IR with ``compile_ir`` (what the CLI prints), checks
the entry's parameter count with ``cuFuncGetParamInfo``, launches it under
the meta geometry with outputs zero-filled, and compares the outputs with the
CPU oracle at the fixture's bar.  One case also goes through the CLI itself.
"""

from __future__ import annotations

import ctypes
import subprocess
import sys

import numpy as np
import pytest

from conftest import CASES, REPO, small_cases

pytestmark = pytest.mark.gpu


def _drv():
    from cuda.bindings import driver
    return driver


def _ok(res):
    """The value(s) of a cuda-python driver call, after checking its status."""
    res = res if isinstance(res, tuple) else (res,)
    assert res[0] == _drv().CUresult.CUDA_SUCCESS, res[0]
    return res[1] if len(res) == 2 else res[1:]


@pytest.fixture(scope="module")
def context(cuda_device):
    import torch
    torch.cuda.init()
    torch.zeros(1, device="cuda")  # torch makes the device's primary context current on this thread
    drv = _drv()
    ctx = _ok(drv.cuCtxGetCurrent())
    if int(ctx) == 0:
        dev = _ok(drv.cuDeviceGet(0))
        ctx = _ok(drv.cuDevicePrimaryCtxRetain(dev))
        _ok(drv.cuCtxSetCurrent(ctx))
    return ctx


def _launch_foreign(ptx: str, spec, bufs: dict) -> None:
    """Load ``ptx`` and launch ``spec.entry`` as the reference's runner did."""
    import torch
    drv = _drv()
    mod = _ok(drv.cuModuleLoadData(ptx.encode("ascii") + b"\0"))
    try:
        fn = _ok(drv.cuModuleGetFunction(mod, spec.entry.encode()))
        nparams = 0
        while True:
            err, _, _ = drv.cuFuncGetParamInfo(fn, nparams)
            if err != drv.CUresult.CUDA_SUCCESS:
                break
            nparams += 1
        assert nparams == len(spec.arg_order), f"entry takes {nparams} parameters, arg_order has {len(spec.arg_order)}"
        vals, types = [], []
        for name in spec.arg_order:
            a = spec.args.get(name, {})
            if a.get("scalar"):
                if (a.get("dtype") or "f32") == "f32":
                    vals.append(float(a["value"]))
                    types.append(ctypes.c_float)
                else:
                    vals.append(int(a["value"]))
                    types.append(ctypes.c_int)
            else:
                vals.append(bufs[name].data_ptr())
                types.append(ctypes.c_void_p)
        k = spec.kernel
        g = (list(k["grid"]) + [1, 1])[:3]
        b = (list(k["block"]) + [1, 1])[:3]
        smem = int(k.get("smem_bytes") or 0)
        if smem > 48 * 1024:
            _ok(drv.cuFuncSetAttribute(fn, drv.CUfunction_attribute.CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES,
                                       smem))
        stream = torch.cuda.current_stream().cuda_stream
        _ok(drv.cuLaunchKernel(fn, *g, *b, smem, stream, (tuple(vals), tuple(types)), 0))
        torch.cuda.synchronize()
    finally:
        _ok(drv.cuModuleUnload(mod))


def _check(cid, spec, got: dict, want: dict) -> None:
    import interp
    check = spec.meta.get("check", {})
    kind = check.get("kind", "ulp")
    for name in spec.outputs:
        o, q = got[name].reshape(-1), want[name].reshape(-1)
        if kind == "ulp":
            crit = check.get("oracle", {"ulp": 0})
            ok, why = interp.within(o, q, crit if "ulp" not in crit else {"ulp": crit["ulp"] + check.get("ulp", 1)})
            assert ok, f"{cid}.{name}: drop-in entry vs oracle: {why}"
        elif kind == "exact":
            assert np.array_equal(o, q), f"{cid}.{name}"
        else:
            np.testing.assert_allclose(o, q, rtol=check.get("rtol", 1e-5), atol=check.get("atol", 1e-5),
                                       err_msg=f"{cid}.{name}: drop-in entry vs oracle")


def _buffers(spec, inputs: dict) -> dict:
    import torch
    from emmy_ptx_compiler_b200 import harness
    bufs = {}
    for name in spec.arg_order:
        a = spec.args.get(name, {})
        if a.get("scalar"):
            continue
        dt = a.get("dtype") or "f32"
        if a.get("output"):
            tdt = getattr(torch, harness.TORCH_DTYPES.get(dt, "float32"))
            bufs[name] = torch.zeros(tuple(a.get("shape") or ()) or (1,), dtype=tdt, device="cuda")
        else:
            bufs[name] = harness.to_device(inputs[name], dt, 0)
    return bufs


@pytest.mark.parametrize("cid", small_cases())
def test_cli_ptx_under_the_reference_launch(cid, context):
    import interp
    from emmy_ptx_compiler_b200 import compiler, harness
    spec = harness.load_case(CASES / cid)
    want, inputs = interp.run_case(CASES / cid)
    ptx = compiler.compile_ir(spec.ir_path)
    bufs = _buffers(spec, inputs)
    _launch_foreign(ptx, spec, bufs)
    got = {n: harness.from_device(bufs[n]) for n in spec.outputs}
    _check(cid, spec, got, want)


@pytest.mark.parametrize("cid", ["c2_gelu_64x1000", "c5_gemm_200x136x300", "f_rmsnorm_33x130"])
def test_the_cli_itself(cid, context):
    import interp
    from emmy_ptx_compiler_b200 import harness
    spec = harness.load_case(CASES / cid)
    p = subprocess.run([sys.executable, str(REPO / "compile.py"), str(spec.ir_path)], capture_output=True,
                       text=True, timeout=600, cwd=REPO)
    assert p.returncode == 0, p.stderr[-2000:]
    want, inputs = interp.run_case(CASES / cid)
    bufs = _buffers(spec, inputs)
    _launch_foreign(p.stdout, spec, bufs)
    _check(cid, spec, {n: harness.from_device(bufs[n]) for n in spec.outputs}, want)
