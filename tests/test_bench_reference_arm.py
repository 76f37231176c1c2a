"""bench.py's reference arm on the CPU: the JSON line the round-end driver parses.

`bench.py --impl reference` times the reference's own CPU algorithm (the oracle's
restatement) on the host cores, rank 0 only.  These tests run its two small workloads
(config 1's legacy batch and a sample of config 4's migration copy loop) and check the
line's keys and the zero-copy `e2e` object, and that a rank other than 0 exits 0 without
printing anything (under torchrun only rank 0 reports).
"""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
KEYS = ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
        "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e")


def _run(args, env_extra=None):
    env = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK")}
    env.update(env_extra or {})
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", *args], cwd=ROOT, env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    return [l for l in r.stdout.splitlines() if l.strip()]


@pytest.mark.parametrize("workload,unit", [("config1", "tokens/s"), ("migrate", "GB/s")])
def test_reference_line(workload, unit):
    lines = _run(["--workload", workload, "--steps", "1", "--warmup", "0"])
    assert len(lines) == 1, lines
    d = json.loads(lines[0])
    for k in KEYS:
        assert k in d, k
    assert d["impl"] == "reference"
    assert d["unit"] == unit and d["value"] > 0 and d["ms_per_step"] > 0
    assert d["higher_is_better"] is True and d["vs_baseline"] is None
    assert d["config"]["workload"]
    cb = d["cpu_baseline"]
    assert set(cb) == {"value", "unit", "cores", "kind", "sample"}
    assert cb["value"] == d["value"] and cb["kind"] == "port" and cb["cores"] >= 1
    assert d["e2e"] == {"value": d["value"], "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_other_ranks_print_nothing():
    assert _run(["--steps", "1", "--warmup", "0"], {"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"}) == []
