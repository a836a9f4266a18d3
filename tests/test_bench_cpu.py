"""bench.py's CPU-side contract (no GPU): the reference arm prints one JSON
line with the fields the driver reads, for a throughput config and for the
latency config, and non-zero ranks print nothing."""

from __future__ import annotations

import json
import os
import subprocess
import sys

import pytest

from conftest import REPO


def _run(*args, env_extra=None):
    env = dict(os.environ, **(env_extra or {}))
    p = subprocess.run([sys.executable, str(REPO / "bench.py"), *args], capture_output=True, text=True,
                       timeout=600, env=env, cwd=REPO)
    assert p.returncode == 0, p.stderr[-2000:]
    return [ln for ln in p.stdout.splitlines() if ln.strip()]


@pytest.mark.parametrize("config,higher", [("c2", True), ("c1", False), ("a_attn", True), ("f_softmax", True)])
def test_reference_arm_line(config, higher):
    lines = _run("--impl", "reference", "--config", config, "--steps", "2", "--warmup", "1")
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["higher_is_better"] is higher
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "scaling", "dtype",
                "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["value"] > 0 and d["e2e"]["value"] == d["value"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["warmup"] >= 3          # the contract's minimum, whatever was asked


def test_reference_arm_prints_on_rank_zero_only():
    assert _run("--impl", "reference", "--steps", "2", "--warmup", "1",
                env_extra={"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"}) == []
