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


def test_roofline_block_from_stage_times():
    """The bench's per-stage rooflines from fabricated stage times (no GPU): the dominant
    stage's DRAM traffic comes from the committed ncu summary for that model and length
    only, and a fused o_proj stage (no separate Add+RMSNorm) says what it includes."""
    sys.path.insert(0, str(REPO))
    import bench
    from kernrelay_b200 import model_gen
    cfg = model_gen.CONFIGS["qwen2.5-7b"]
    pk = {"tflops_sustained": 1400.0, "hbm_gbs": 6500.0, "source": "test"}
    st = {"qkv": 2400.0, "attention": 1900.0, "o": 2500.0, "gateup": 12200.0, "addnorm": 0.0,
          "embed": 30.0, "lm_head": 1700.0, "relay": 8100.0}
    roof, stages = bench.roofline_block(cfg, 2048, 1, 0, {"stage_us": st}, pk, 770.0,
                                        "qwen2.5-7b")
    assert roof["kernel"] == "gateup" and roof["bound"] == "tensor"
    assert roof["traffic"] == bench.traffic_for("qwen2.5-7b", 2048, "gateup", 1) > 0
    assert 0.8 < roof["frac"] < 1.0
    assert "includes" in stages["o"] and "addnorm" not in stages
    roof8, _ = bench.roofline_block(cfg, 4096, 1, 0, {"stage_us": st}, pk, 770.0, "qwen3-vl-8b")
    assert roof8["traffic"] is None   # no capture for that model and length
    st2 = dict(st, addnorm=700.0)
    _, stages2 = bench.roofline_block(cfg, 2048, 1, 0, {"stage_us": st2}, pk, 770.0)
    assert "includes" not in stages2["o"] and stages2["addnorm"]["unit"] == "GB/s"
