"""CPU: the benchmark's reference arm (bench.py --impl reference) keeps the JSON-line
contract the round driver reads: the metric, unit and config of the native arm, a
cpu_baseline describing the run, and an end-to-end object with no host<->device
bytes; under torchrun only rank 0 prints."""
from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _run(env_extra: dict[str, str]) -> subprocess.CompletedProcess:
    env = dict(os.environ, **env_extra)
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                           "--steps", "1", "--warmup", "1"], cwd=ROOT, env=env,
                          capture_output=True, text=True, timeout=600)


def test_reference_arm_prints_one_contract_line(oracle):
    res = _run({})
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [l for l in res.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == "complete games/s per box (3x512 MLP self-play)"
    assert d["unit"] == "games/s" and d["higher_is_better"] is True and d["scaling"] == "weak"
    assert (d["n_gpus"], d["steps"], d["warmup"]) == (1, 1, 1)
    assert d["value"] > 0 and d["ms_per_step"] > 0 and d["vs_baseline"] is None
    assert d["config"]["workload"] == "config3-ppo-selfplay-512x3"
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] == "reference" and cb["cores"] >= 1
    assert cb["unit"] == "games/s" and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "games/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_quietly():
    res = _run({"WORLD_SIZE": "2", "RANK": "1", "LOCAL_RANK": "1"})
    assert res.returncode == 0, res.stderr[-2000:]
    assert not [l for l in res.stdout.splitlines() if l.startswith("{")]
