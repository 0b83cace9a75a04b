"""Time schedules through kr_plan_run: unsplit (A) against split (B) groups, per launch mode.

    python -m kernrelay_b200.plan_bench --plans tests/golden/plans/full \\
        --dags f02_mm_gelu_c4,e9_two_waves --modes direct,graph --devices 0 --out r.json

For each DAG and mode prints one JSON line: host p50 (the reference's p50_us, wall time
of enqueue + completion), device p50 (CUDA events around the schedule's lanes), the
B-over-A speedup of each, and the matmul work as TFLOP/s of device time.  Schedules with
nranks > 1 run on the first nranks ids of --devices.
"""
import argparse
import json
import tempfile
from pathlib import Path

from kernrelay_b200 import libapi


def matmul_flops(sched):
    return sum(2.0 * n["rows"] * n["k"] * n["n"] for n in sched["nodes"] if n["op"] == "matmul")


def run_one(path, devices, mode, iters, warmup):
    with tempfile.TemporaryDirectory() as td:
        r = libapi.plan_run(path, devices=devices, mode=mode, iters=iters, warmup=warmup,
                            out_json=Path(td) / "o.json")
    if r.get("_rc") != 0:
        raise RuntimeError(f"{path} {mode}: {r.get('error')}")
    return r


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--plans", required=True, help="directory holding <dag>_a.json / <dag>_b.json")
    ap.add_argument("--dags", required=True)
    ap.add_argument("--modes", default="direct,graph")
    ap.add_argument("--devices", default="0")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--out")
    args = ap.parse_args()
    rows = []
    for dag in args.dags.split(","):
        for mode in args.modes.split(","):
            line = {"dag": dag, "mode": mode}
            for g in ("a", "b"):
                path = Path(args.plans) / f"{dag}_{g}.json"
                sched = json.loads(path.read_text(encoding="utf-8"))
                devs = ",".join(args.devices.split(",")[:int(sched.get("nranks", 1))])
                r = run_one(path, devs, mode, args.iters, args.warmup)
                line[g] = {"p50_us": r["p50_us"], "device_p50_us": r["device_p50_us"],
                           "checksum": r["checksum"], "tasks": sum(len(v) for v in sched["streams"].values())}
                flops = matmul_flops(sched)
                if flops:
                    line[g]["matmul_tflops"] = flops / (r["device_p50_us"] * 1e-6) / 1e12
            line["speedup_host"] = line["a"]["p50_us"] / line["b"]["p50_us"]
            line["speedup_device"] = line["a"]["device_p50_us"] / line["b"]["device_p50_us"]
            print(json.dumps(line), flush=True)
            rows.append(line)
    if args.out:
        Path(args.out).write_text(json.dumps(rows, indent=1), encoding="utf-8")


if __name__ == "__main__":
    main()
