"""bench.py's reference arm runs on the host cores and needs no GPU: rank 0
prints one JSON line with the contract's keys, tagged "impl": "reference", whose
cpu_baseline and e2e records describe the same run; any other rank of a
torchrun launch exits 0 without work or output."""
import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
CMD = [sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "3"]


def test_reference_arm_prints_one_contract_line():
    res = subprocess.run(CMD, cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [line for line in res.stdout.splitlines() if line.strip()]
    assert len(lines) == 1, res.stdout
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config"):
        assert key in d, key
    assert d["impl"] == "reference" and d["steps"] == 1 and d["warmup"] >= 3 and d["value"] > 0
    assert d["unit"] == "GB/s" and d["higher_is_better"] is True
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["unit"] == d["unit"] and cb["kind"] in ("port", "reference")
    assert cb["cores"] >= 1 and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_quietly():
    env = dict(os.environ, RANK="1", LOCAL_RANK="1", WORLD_SIZE="2")
    res = subprocess.run(CMD, cwd=ROOT, capture_output=True, text=True, timeout=300, env=env)
    assert res.returncode == 0, res.stderr[-2000:]
    assert res.stdout.strip() == ""
