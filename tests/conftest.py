"""Shared test configuration.

* ``gpu`` marks tests that need a B200 (``-m gpu``); everything else runs on
  CPU in a few minutes.
* ``oracle/`` (the CPU restatement of the reference) and the fixture index
  are importable from every test.
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
GOLDEN = REPO / "tests" / "golden"
CASES = GOLDEN / "cases"
# the reference checkout (read-only), by default beside this repository; tests that need it skip without it
REFERENCE = Path(os.environ.get("EMMY_REFERENCE", str(Path(__file__).resolve().parents[2] / "reference")))

for p in (REPO, REPO / "oracle"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100a GPU (run with -m gpu)")


def case_index() -> list[dict]:
    return json.loads((CASES / "INDEX.json").read_text())["cases"]


def small_cases(family: str | None = None) -> list[str]:
    out = []
    for c in case_index():
        if c["id"].endswith("_full") or "2p28" in c["id"] or "_prof_" in c["id"] or "_bench_" in c["id"]:
            continue
        if family and c["family"] != family:
            continue
        out.append(c["id"])
    return out


@pytest.fixture(scope="session")
def cuda_device():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from emmy_ptx_compiler_b200 import runtime
    runtime.init(0)
    return 0
