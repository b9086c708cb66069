"""The JSON line bench.py prints for the reference arm, checked on the CPU: the driver launches
`bench.py --impl reference` beside the B200 arm and reads one line from rank 0 (the other ranks of a
torchrun launch print nothing and exit 0).  The B200 arm's line has the same keys plus the roofline,
e2e copies and clocks; it needs a GPU and runs in the round-end bench."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(env_extra=None):
    env = dict(os.environ)
    env.pop("RANK", None)
    env.pop("WORLD_SIZE", None)
    env.update(env_extra or {})
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "3",
                           "--warmup", "3"], capture_output=True, text=True, env=env, cwd=ROOT, timeout=600)


@pytest.mark.timeout(600)
def test_reference_arm_prints_one_contract_line():
    done = _run()
    assert done.returncode == 0, done.stderr[-2000:]
    lines = [ln for ln in done.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, done.stdout[-2000:]
    line = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["unit"] == "GB/s" and line["higher_is_better"] is True
    assert line["steps"] == 3 and line["warmup"] == 3 and line["value"] > 0
    assert line["config"]["workload"].startswith("softmax+rmsnorm bf16 [4096,4096]")
    base = line["cpu_baseline"]
    assert base["kind"] in ("port", "reference") and base["cores"] >= 1 and base["value"] == line["value"]
    assert isinstance(base["sample"], str) and base["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


@pytest.mark.timeout(120)
def test_reference_arm_other_ranks_exit_quietly():
    done = _run({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert done.returncode == 0, done.stderr[-2000:]
    assert not [ln for ln in done.stdout.splitlines() if ln.startswith("{")]
