"""bench.py's reference arm (CPU only): one JSON line on stdout with the contract's keys, and
nothing from ranks other than 0."""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

import oracle

ROOT = Path(__file__).resolve().parents[1]
KEYS = {"impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
        "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"}


def _run(env_extra):
    env = {**os.environ, **env_extra}
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                           "--warmup", "3"], capture_output=True, text=True, env=env, cwd=ROOT, timeout=600)


@pytest.mark.skipif(oracle.available_reference() is None, reason="reference CPU kernel not built here")
def test_reference_arm_prints_one_contract_line():
    res = _run({"RANK": "0", "WORLD_SIZE": "1"})
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [line for line in res.stdout.splitlines() if line.strip()]
    assert len(lines) == 1
    record = json.loads(lines[0])
    assert KEYS <= set(record)
    assert record["impl"] == "reference" and record["value"] > 0 and record["higher_is_better"] is True
    assert record["e2e"]["h2d_bytes_per_step"] == 0 and record["cpu_baseline"]["kind"] == "reference"
    assert record["cpu_baseline"]["cores"] >= 1


def test_reference_arm_other_ranks_print_nothing():
    res = _run({"RANK": "1", "WORLD_SIZE": "2"})
    assert res.returncode == 0, res.stderr[-2000:]
    assert res.stdout.strip() == ""
