"""``bench.py``'s output contract, checked on a CPU-only host through its reference arm (the
reference's CPU chain needs no GPU): exactly one JSON line on stdout with the keys and units its
readers expect, the metric of BASELINE.json, and silence from ranks other than 0."""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def _run(extra_env=None):
    env = dict(os.environ)
    env.pop("RANK", None)
    env.pop("WORLD_SIZE", None)
    env.pop("LOCAL_RANK", None)
    env.update(extra_env or {})
    return subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--workload",
                           "minigpt_6l_384", "--steps", "1", "--warmup", "1"], cwd=ROOT, env=env,
                          capture_output=True, text=True, timeout=600)


def test_reference_arm_prints_one_contract_line():
    res = _run()
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [ln for ln in res.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, res.stdout
    d = json.loads(lines[0])
    baseline = json.loads((ROOT / "BASELINE.json").read_text())
    assert d["metric"] == baseline["metric"]
    assert d["impl"] == "reference"
    for key in ("value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e",
                "gpu_launches"):
        assert key in d, key
    assert d["unit"] == "Gparams/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert (d["n_gpus"], d["steps"], d["warmup"]) == (1, 1, 1)
    assert d["vs_baseline"] is None
    assert "workload" in d["config"]
    cpu = d["cpu_baseline"]
    assert cpu["kind"] == "reference" and cpu["cores"] >= 1 and cpu["value"] == d["value"]
    assert cpu["unit"] == d["unit"] and cpu["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
    assert d["gpu_launches"] == 0


def test_reference_arm_is_silent_on_other_ranks():
    res = _run({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert res.returncode == 0, res.stderr[-2000:]
    assert res.stdout.strip() == ""
