#!/usr/bin/env python3
"""Capture golden vectors from the reference compiler's PTX run on a B200.

    python tests/golden/capture_ref_outputs.py OUT_DIR

For every small fixture that has a reference PTX (``ref.ptx``, or
``ref_f32/ref.ptx`` for bf16 GEMMs), generate the fixture's seeded inputs
(the meta ``args`` recipes), launch the reference module through
libemmy_b200 under the meta.json geometry - as the reference's runner did -
and store the outputs (first 65536 elements of each) in ``OUT_DIR/<case>.npz``
plus ``OUT_DIR/INDEX.json``.  The committed copy lives in
tests/golden/ref_outputs/ and pins the CPU oracle (tests/test_oracle_cpu.py).
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REPO / "oracle"))

LIMIT = 65536
APPROX_OPS = ("exp", "tanh", "sigmoid", "silu", "log", "rsqrt", "exp2", "log2", "pow")


def main() -> int:
    import torch

    import interp
    from emmy_ptx_compiler_b200 import harness, runtime

    out_dir = Path(sys.argv[1])
    out_dir.mkdir(parents=True, exist_ok=True)
    runtime.init(0)
    index = json.loads((HERE / "cases" / "INDEX.json").read_text())["cases"]
    done = {}
    for rec in index:
        cid = rec["id"]
        if cid.endswith("_full") or "2p28" in cid or "_prof_" in cid or "_bench_" in cid:
            continue
        d = HERE / "cases" / cid
        ref_dir = d if (d / "ref.ptx").is_file() else (d / "ref_f32" if (d / "ref_f32" / "ref.ptx").is_file() else None)
        if ref_dir is None:
            continue
        spec = harness.load_case(ref_dir)
        kop, meta, mk, shapes, dtypes = interp.load_case(d)
        inputs = interp.make_inputs(mk, shapes, dtypes)
        mod = harness.ForeignModule((ref_dir / "ref.ptx").read_bytes(), spec, 0)
        bufs = {}
        for name in spec.arg_order:
            a = spec.args[name]
            if a.get("output"):
                bufs[name] = torch.zeros(tuple(a["shape"]) or (1,), dtype=torch.float32, device="cuda:0")
            else:
                bufs[name] = harness.to_device(inputs[name], "f32", 0)
        mod.run(bufs)
        torch.cuda.synchronize()
        outs = {n: harness.from_device(bufs[n]).reshape(-1)[:LIMIT] for n in spec.outputs}
        mod.module.close()
        np.savez(out_dir / f"{cid}.npz", **outs)
        text = (next(ref_dir.glob("*.ir.json"))).read_text()
        approx = any(f"name='{op}'" in text for op in APPROX_OPS)
        done[cid] = {"case_dir": str(ref_dir.relative_to(HERE / "cases")), "outputs": list(outs),
                     "approx": approx, "elements": {k: int(v.size) for k, v in outs.items()}}
        print(f"captured {cid}", file=sys.stderr)
    (out_dir / "INDEX.json").write_text(json.dumps({
        "note": "outputs of the reference compiler's PTX (tests/golden/cases/*/ref.ptx) launched on a "
                "B200 by tests/golden/capture_ref_outputs.py, inputs from the fixture meta recipes",
        "cases": done}, indent=1) + "\n")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
