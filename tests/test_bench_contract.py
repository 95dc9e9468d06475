"""bench.py's driver contract on the CPU: `--impl reference` prints one JSON line with the
reference arm's keys (the reference's own CPU path on the host cores: invokerl imported from
baseline/_ref, or the oracle's restatement when that copy is absent), and the end-to-end workload
prints its `unavailable` line instead."""

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def _run(*args, env_extra=None):
    env = dict(os.environ, **(env_extra or {}))
    res = subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True, text=True,
                         timeout=600, env=env, cwd=ROOT)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [ln for ln in res.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, res.stdout
    return json.loads(lines[0])


def test_reference_arm_prints_one_json_line():
    d = _run("--impl", "reference", "--workload", "grpo", "--steps", "1", "--warmup", "1")
    assert d["impl"] == "reference"
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "config",
              "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["value"] > 0 and d["higher_is_better"] is True
    have_ref = (ROOT / "baseline" / "_ref" / "invokerl" / "policy.py").exists()
    assert d["cpu_baseline"]["kind"] == ("reference" if have_ref else "port")
    assert d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["value"] == d["value"]


def test_end_to_end_workload_reference_arm_is_unavailable():
    d = _run("--impl", "reference", "--workload", "e2e-0.6b", "--steps", "1", "--warmup", "1")
    assert d["impl"] == "reference" and "unavailable" in d
