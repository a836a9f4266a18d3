"""The test shim for the absent ``emmy`` package is faithful enough for the
reference compiler: its own unit tests pass against it (CPU only; skipped
where the reference checkout is not mounted)."""

from __future__ import annotations

import os
import subprocess
import sys

import pytest

from conftest import REFERENCE, REPO

MODULES = ["test_collective_guard", "test_extra_isa", "test_no_hardcode", "test_open_set", "test_peepholes"]


@pytest.mark.skipif(not (REFERENCE / "compile.py").is_file(), reason="reference checkout not mounted")
def test_reference_unit_tests_pass_on_the_shim():
    env = dict(os.environ, PYTHONDONTWRITEBYTECODE="1",
               PYTHONPATH=f"{REPO / 'oracle' / 'emmy_shim'}:{REFERENCE}")
    p = subprocess.run([sys.executable, "-m", "unittest", *MODULES], cwd=REFERENCE / "tests", env=env,
                       capture_output=True, text=True, timeout=300)
    assert p.returncode == 0, p.stderr[-3000:]
    assert "OK" in p.stderr


def test_fixture_bodies_evaluate_in_the_shim():
    sys.path.insert(0, str(REPO / "oracle" / "emmy_shim"))
    import json
    from emmy._core import Graph, KernelOp
    from conftest import CASES, case_index
    for rec in case_index():
        raw = json.loads((CASES / rec["ir"]).read_text())
        g = Graph.from_dict(raw)
        kop = next(n.op for n in g.nodes.values() if isinstance(n.op, KernelOp))
        assert kop.name == rec["entry"]
