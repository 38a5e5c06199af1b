"""bench.py's reference arm (the reference's own CPU decode path, from the unmodified install in
baseline/_ref) as the benchmark driver runs it: one JSON line with the metric, the config the GPU arm
prints, the CPU baseline that produced it and an end-to-end entry without device copies; under a
multi-rank launch only rank 0 reports."""

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
    import bench

    B, distinct, arena = bench.batched_plan(bench.WORKLOADS["batched"], 1)
    assert d["config"] == bench.batched_config(bench.WORKLOADS["batched"], 1, B, distinct, arena)
    assert d["config"]["kv_pool_gb_per_gpu"] > 20 and d["config"]["distinct_layer_stores"] == 28
    cb = d["cpu_baseline"]
    kind = "reference" if (ROOT / "baseline" / "_ref" / "anchorkv").exists() else "port"
    assert cb["value"] == d["value"] and cb["unit"] == "GB/s" and cb["kind"] == kind and cb["cores"] >= 1
    assert "decode calls" in cb["sample"]
    if kind == "reference":
        assert "PagedLayer (baseline/_ref, unmodified" in cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_long_context_reference_arm_prints_the_long_config():
    d = _bench("--impl", "reference", "--workload", "long", "--steps", "3", "--warmup", "3",
               "--cpu-seconds", "0.5")[0]
    import bench

    assert d["config"] == bench.long_config(bench.LONG, 1) and d["scaling"] == "strong"
    assert d["config"]["context_tokens"] == 1 << 20 and d["value"] > 0


def test_reference_arm_reports_on_rank_zero_only():
    env = {"RANK": "1", "LOCAL_RANK": "1", "WORLD_SIZE": "2"}
    assert _bench("--impl", "reference", "--steps", "3", "--warmup", "3", "--cpu-seconds", "0.5", env=env) == []


def test_warmup_below_three_is_refused():
    proc = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--warmup", "2"], cwd=ROOT,
                          capture_output=True, text=True, timeout=120)
    assert proc.returncode != 0 and "warmup" in proc.stderr
