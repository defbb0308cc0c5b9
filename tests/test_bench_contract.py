"""CPU checks of bench.py's output contract through its reference arm (the
CPU restatement timed on the host): one JSON line on rank 0 with the keys
the round driver reads, and no output from the other ranks."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def run_bench(env_extra, *args):
    env = dict(os.environ, **env_extra)
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args],
                          cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)


def test_reference_arm_line():
    r = run_bench({"RANK": "0", "WORLD_SIZE": "1"}, "--impl", "reference", "--steps", "3",
                  "--warmup", "3")
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == "decode cache-path us/token/layer"
    assert d["unit"] == "us" and d["higher_is_better"] is False
    assert d["value"] > 0 and d["steps"] == 3 and d["warmup"] == 3
    assert d["config"]["name"] == "stack" and d["config"]["sequences"] == 64
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == d["value"]
    e = d["e2e"]
    assert e["value"] == d["value"] and e["unit"] == d["unit"]
    assert e["h2d_bytes_per_step"] == 0 and e["d2h_bytes_per_step"] == 0


def test_reference_arm_other_ranks_silent():
    r = run_bench({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"}, "--impl", "reference",
                  "--gpus", "2", "--steps", "3", "--warmup", "3")
    assert r.returncode == 0, r.stderr[-2000:]
    assert not [ln for ln in r.stdout.splitlines() if ln.startswith("{")], r.stdout
