"""bench.py's CPU-side contract: the reference arm's JSON line (host cores, no GPU), rank 0
alone printing under torchrun, and the world-size check of our arm."""
import json
import os
import subprocess
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]


def _bench(args, env_extra):
    env = dict(os.environ, **env_extra)
    return subprocess.run([sys.executable, str(REPO / "bench.py")] + args, cwd=REPO, env=env,
                          capture_output=True, text=True, timeout=600)


def test_reference_arm_prints_one_contract_line():
    """Each reference step is a complete prefill that is really timed: the steps times
    ms_per_step fit inside the process's own wall time (no extrapolated steps)."""
    import time
    t0 = time.time()
    p = _bench(["--impl", "reference", "--steps", "2", "--warmup", "1", "--seq", "256",
                "--config", "qwen2.5-0.5b"], {"RANK": "0", "WORLD_SIZE": "1"})
    wall = time.time() - t0
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [l for l in p.stdout.splitlines() if l.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0 and d["higher_is_better"] is True
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
    assert d["steps"] == 2 and d["warmup"] == 1
    assert d["steps"] * d["ms_per_step"] / 1e3 <= wall
    assert abs(d["steps"] * d["ms_per_step"] / 1e3 - d["timed_wall_s"]) < 0.05
    assert d["config"]["workload"] == "qwen2.5-0.5b prefill S=256 batch 1"


def test_reference_arm_other_ranks_exit_quietly():
    p = _bench(["--impl", "reference", "--gpus", "2"], {"RANK": "1", "WORLD_SIZE": "2"})
    assert p.returncode == 0 and p.stdout.strip() == ""


def test_our_arm_checks_world_size():
    p = _bench(["--gpus", "2"], {"RANK": "0", "WORLD_SIZE": "1"})
    assert p.returncode != 0 and "WORLD_SIZE=1" in (p.stderr + p.stdout)
