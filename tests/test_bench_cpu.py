"""bench.py's reference arm on the CPU: zpu's CPU jit path (the oracle port)
timed on the host cores, printed as one JSON line with the keys the bench
contract names; under a multi-rank launch only rank 0 prints."""
import json
import os
import subprocess
import sys

from tests.helpers import ROOT

KEYS = ["impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
        "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"]


def run_bench(args, env_extra=None):
    env = dict(os.environ)
    env.update(env_extra or {})
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py")] + args, cwd=ROOT, env=env,
                          capture_output=True, text=True, timeout=900)


def json_lines(out):
    return [json.loads(line) for line in out.splitlines() if line.startswith("{")]


def test_reference_arm_prints_one_contract_line():
    r = run_bench(["--impl", "reference", "--steps", "1", "--warmup", "0"])
    assert r.returncode == 0, r.stderr[-2000:]
    lines = json_lines(r.stdout)
    assert len(lines) == 1, r.stdout
    d = lines[0]
    missing = [k for k in KEYS if k not in d]
    assert not missing, missing
    assert d["impl"] == "reference" and d["unit"] == "GB/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["steps"] == 1 and d["n_gpus"] == 1
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["value"] == d["value"]
    assert d["cpu_baseline"]["cores"] >= 1 and d["cpu_baseline"]["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["config"]["workload"]


def test_reference_arm_prints_on_rank_zero_only():
    r = run_bench(["--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "0"],
                  {"RANK": "1", "LOCAL_RANK": "1", "WORLD_SIZE": "2"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert json_lines(r.stdout) == []
