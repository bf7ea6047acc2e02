"""bench.py's reference arm (the lab's CPU path, restated in C), on CPU: one
JSON line with the benchmark contract's keys, exactly --steps timed steps
after --warmup untimed ones, and silence on every rank but 0."""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _run(extra_env: dict, *args: str) -> subprocess.CompletedProcess:
    env = dict(os.environ, **extra_env)
    env.pop("CUDA_VISIBLE_DEVICES", None)
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", *args],
                          cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)


def test_reference_arm_line():
    r = _run({}, "--steps", "2", "--warmup", "3")
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference"
    assert (d["steps"], d["warmup"], d["n_gpus"]) == (2, 3, 1)
    assert d["higher_is_better"] is True and d["vs_baseline"] is None and d["value"] > 0
    assert d["config"]["workload"] == "config1_decode_batch32"
    assert abs(d["ms_per_step"] - 1000.0 * d["config"]["tokens_per_step"] / d["value"]) < 1e-2
    cpu = d["cpu_baseline"]
    assert cpu["value"] == d["value"] and cpu["unit"] == d["unit"] and cpu["kind"] == "port"
    assert cpu["cores"] >= 1 and cpu["sample"].startswith("2 steps")
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_quietly():
    r = _run({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"}, "--gpus", "2", "--steps", "2",
             "--warmup", "3")
    assert r.returncode == 0, r.stderr[-2000:]
    assert not [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
