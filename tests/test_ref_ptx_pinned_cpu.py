"""Every committed ``ref.ptx`` is exactly what the unmodified reference
compiler prints for the committed IR next to it.

The GPU parity chain rests on these files: the golden vectors under
``tests/golden/ref_outputs`` are outputs of ``ref.ptx`` run on a B200, and
the oracle is pinned to those vectors.  This test recompiles each fixture's
IR with the reference's own ``compile_bundle`` (compile.py:3168-3215, through
the ``emmy`` test shim) and requires byte equality with the committed PTX.
CPU only; skipped where the reference checkout is not mounted.
"""

from __future__ import annotations

import json
import os
import subprocess
import sys

import pytest

from conftest import CASES, REFERENCE, REPO, case_index

_DRIVER = r"""
import json, sys
from pathlib import Path
sys.dont_write_bytecode = True
import compile as ref
cases = Path(sys.argv[1])
bad, seen = [], 0
for rel in json.loads(sys.stdin.read()):
    ptx_path = cases / rel
    ir = next(ptx_path.parent.glob("*.ir.json"))
    got = ref.compile_bundle(ir)["ptx"]
    seen += 1
    if got.encode() != ptx_path.read_bytes():
        bad.append(rel)
print(json.dumps({"checked": seen, "differ": bad}))
"""


def _ref_ptx_files() -> list[str]:
    out = []
    for rec in case_index():
        if rec.get("ref_ptx"):
            out.append(rec["ref_ptx"])
    return out


def test_every_case_with_reference_ptx_is_indexed():
    indexed = set(_ref_ptx_files())
    on_disk = {str(p.relative_to(CASES)) for p in CASES.rglob("ref.ptx")}
    assert on_disk == indexed, sorted(on_disk ^ indexed)


@pytest.mark.skipif(not (REFERENCE / "compile.py").is_file(), reason="reference checkout not mounted")
def test_ref_ptx_is_the_reference_compilers_output():
    files = _ref_ptx_files()
    assert len(files) > 50
    env = dict(os.environ, PYTHONDONTWRITEBYTECODE="1",
               PYTHONPATH=f"{REPO / 'oracle' / 'emmy_shim'}:{REFERENCE}")
    p = subprocess.run([sys.executable, "-c", _DRIVER, str(CASES)], input=json.dumps(files), env=env,
                       capture_output=True, text=True, timeout=600, cwd=str(REFERENCE))
    assert p.returncode == 0, p.stderr[-3000:]
    res = json.loads(p.stdout.strip().splitlines()[-1])
    assert res["checked"] == len(files)
    assert res["differ"] == [], f"ref.ptx differs from the reference compiler's output: {res['differ']}"
