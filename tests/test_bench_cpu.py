"""bench.py's reference arm on the host (no GPU): the JSON line the driver reads, its keys and their meaning, and the
torchrun rule that only rank 0 runs and prints it. The timed work is the oracle port of the reference's CPU path."""

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def run_bench(*args, env_extra=None, timeout=600):
    env = dict(os.environ)
    env.update({"OMP_NUM_THREADS": env.get("OMP_NUM_THREADS", "4")})
    if env_extra:
        env.update(env_extra)
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], cwd=ROOT, env=env, capture_output=True,
                          text=True, timeout=timeout)


def json_lines(out):
    return [json.loads(l) for l in out.splitlines() if l.startswith("{")]


def test_reference_arm_prints_one_contract_line():
    r = run_bench("--impl", "reference", "--steps", "1", "--warmup", "1")
    assert r.returncode == 0, r.stderr[-2000:]
    lines = json_lines(r.stdout)
    assert len(lines) == 1, r.stdout
    d = lines[0]
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["value"] > 0 and d["unit"] == "TOPS" and d["higher_is_better"] is True
    assert d["steps"] == 1 and d["warmup"] >= 3 and d["n_gpus"] == 1
    assert "workload" in d["config"]
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    # the same algorithmic work per step as the GPU arm's job, so the driver's ratio compares like with like
    import bench
    assert d["metric"] == bench.METRIC
    assert d["config"] == bench.job_config(1, d["config"]["rows_per_gpu"])


def test_reference_arm_other_ranks_exit_quietly():
    r = run_bench("--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "1",
                  env_extra={"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"}, timeout=120)
    assert r.returncode == 0, r.stderr[-2000:]
    assert json_lines(r.stdout) == []
