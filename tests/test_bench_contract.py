"""bench.py's reference arm (CPU only) prints one JSON line with the contract
keys; the other ranks of a torchrun launch print nothing."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def run(env_extra):
    env = dict(os.environ, **env_extra)
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "2",
                        "--warmup", "1"], capture_output=True, text=True, timeout=600, env=env, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    return [l for l in r.stdout.splitlines() if l.startswith("{")]


def test_reference_arm_line():
    lines = run({"WORLD_SIZE": "1", "RANK": "0", "LOCAL_RANK": "0"})
    assert len(lines) == 1
    d = json.loads(lines[0])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
              "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference" and d["value"] > 0
    # the driver's step counts, not clamped
    assert d["steps"] == 2 and d["warmup"] == 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["value"] == d["value"]
    assert set(("value", "unit", "cores", "kind", "sample")) <= set(d["cpu_baseline"])


def test_reference_arm_other_ranks_silent():
    assert run({"WORLD_SIZE": "2", "RANK": "1", "LOCAL_RANK": "1"}) == []
