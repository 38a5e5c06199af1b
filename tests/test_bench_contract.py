"""bench.py's reference arm (the reference's CPU decode path, restated with torch CPU ops) as the
benchmark driver runs it: one JSON line with the metric, the CPU baseline that produced it and an
end-to-end entry without device copies; under a multi-rank launch only rank 0 reports."""

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def _bench(*args, env=None):
    e = dict(os.environ, **(env or {}))
    proc = subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], cwd=ROOT, env=e,
                          capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stderr[-2000:]
    return [json.loads(line) for line in proc.stdout.splitlines() if line.startswith("{")]


def test_reference_arm_prints_one_line_with_the_contract_keys():
    lines = _bench("--impl", "reference", "--steps", "3", "--warmup", "3", "--cpu-seconds", "0.5")
    assert len(lines) == 1
    d = lines[0]
    assert d["impl"] == "reference" and d["unit"] == "GB/s" and d["higher_is_better"] is True
    assert d["n_gpus"] == 1 and d["steps"] == 3 and d["warmup"] == 3 and d["value"] > 0
    assert d["metric"].startswith("decode-attn resident-KV GB/s")
    assert d["config"]["workload"].startswith("batched decode") and d["config"]["batch_per_gpu"] == 64
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["unit"] == "GB/s" and cb["kind"] == "port" and cb["cores"] >= 1
    assert "decode calls" in cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_reports_on_rank_zero_only():
    env = {"RANK": "1", "LOCAL_RANK": "1", "WORLD_SIZE": "2"}
    assert _bench("--impl", "reference", "--steps", "3", "--warmup", "3", "--cpu-seconds", "0.5", env=env) == []


def test_warmup_below_three_is_refused():
    proc = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--warmup", "2"], cwd=ROOT,
                          capture_output=True, text=True, timeout=120)
    assert proc.returncode != 0 and "warmup" in proc.stderr
