"""``bench.py --impl reference``: the reference arm runs on the host cores (the oracle port
of the reference's CPU path), so its output contract is checked here without a GPU: one
JSON line with the headline metric, the reference marker, a ``cpu_baseline`` record that
describes the run and an ``e2e`` record with no host-device traffic; under torchrun only
rank 0 runs and prints."""

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(env_extra):
    env = dict(os.environ, **env_extra)
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0"],
                       cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    return [line for line in r.stdout.splitlines() if line.startswith("{")]


def test_reference_arm_prints_one_contract_line():
    lines = _run({"RANK": "0", "WORLD_SIZE": "1", "LOCAL_RANK": "0"})
    assert len(lines) == 1
    rec = json.loads(lines[0])
    assert rec["impl"] == "reference"
    assert rec["metric"].startswith("atom-steps/s") and rec["unit"] == "atom-steps/s"
    assert rec["higher_is_better"] is True and rec["steps"] == 1 and rec["warmup"] == 0
    assert rec["value"] > 0 and rec["ms_per_step"] > 0
    base = rec["cpu_baseline"]
    assert base["kind"] == "port" and base["cores"] >= 1 and base["value"] == rec["value"]
    assert "192-atom" in base["sample"]
    e2e = rec["e2e"]
    assert e2e["value"] == rec["value"] and e2e["unit"] == rec["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    assert "27,648-atom" in rec["config"]["workload"]


def test_reference_arm_other_ranks_exit_without_output():
    assert _run({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"}) == []
