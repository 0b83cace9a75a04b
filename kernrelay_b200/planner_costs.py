"""B200 cost tables for the reference planner, measured through kr_plan_run / kr_qwen_profile_many.

The reference planner (python/kernrelay/planner2.py, class Costs) reads two files:
  * a cost table (configs/planner2_costs.json): launch_us, traffic_gbps, l2_mb,
    event_us, split overheads and "full" = measured time of each op|shape unsplit;
  * split curves (configs/planner_curves.json): for each E1 case, the total time of k
    consecutive tiles for k = 1..K, fitted as total(k) = intercept + slope * (k - 1)
    (planner2.py:130-165 uses slope_us_per_tile, intercept_us and base_best_us).
This module measures both on the local GPUs and writes them in the same formats:

    python -m kernrelay_b200.planner_costs --out-dir kernrelay_b200/configs --devices 0
    python -m kernrelay_b200.planner_costs --out-dir DIR --devices 0,1 --qwen qwen2.5-0.5b

Each curve point is a one-node schedule with k row tasks (column tasks for the "col"
strategy) on one lane, run by kr_plan_run in direct mode; the value is the best device
time of the k back-to-back launches.  Qwen operator costs come from kr_qwen_profile_many
(k = 1 slices of a random-init model of the named architecture).  Collective costs are
measured only when --devices names two or more GPUs.
"""
import argparse
import json
import tempfile
from pathlib import Path

from kernrelay_b200 import libapi

# The reference's E1 curve cases (configs/planner_curves.json): name, op, strategy, shape.
CURVE_CASES = [
    ("mm_mid", "matmul", "row", {"M": 8192, "K": 1024, "N": 2048}),
    ("mm_large", "matmul", "row", {"M": 32768, "K": 1024, "N": 2048}),
    ("mm_24576", "matmul", "row", {"M": 24576, "K": 1024, "N": 2048}),
    ("gelu_large", "gelu", "row", {"rows": 32768, "cols": 2048}),
    ("softmax_large", "softmax", "row", {"rows": 32768, "cols": 2048}),
    ("layernorm_large", "layernorm", "row", {"rows": 32768, "cols": 2048}),
    ("cast_large", "cast", "row", {"rows": 32768, "cols": 2048}),
    ("mm_balanced_col", "matmul", "col", {"M": 65536, "K": 2048, "N": 4096}),
    ("gelu_huge", "gelu", "row", {"rows": 131072, "cols": 4096}),
    ("layernorm_huge", "layernorm", "row", {"rows": 131072, "cols": 4096}),
    ("add_huge", "add", "row", {"rows": 131072, "cols": 4096}),
    ("softmax_huge", "softmax", "row", {"rows": 131072, "cols": 4096}),
    ("cast_huge", "cast", "row", {"rows": 131072, "cols": 4096}),
    ("topk_huge", "topk", "row", {"rows": 8192, "cols": 4096, "k": 128}),
    ("sort_huge", "sort", "row", {"rows": 4096, "cols": 4096}),
    ("embedding_huge", "embedding", "row", {"rows": 65536, "cols": 1024, "vocab": 32000}),
]
KS = (1, 2, 3, 4, 6, 8, 12, 16, 32)

# generic op|shape keys of the reference cost table measured with the plan executor
EXTRA_FULL = [
    ("matmul", {"M": 65536, "K": 2048, "N": 4096}),
]
COMM_FULL = [("allreduce", 2048, 2048), ("allreduce", 32768, 2048), ("allgather", 2048, 2048),
             ("reducescatter", 2048, 2048),
             # the TP layer's exchange (scripts/tp_planner.py: 2048 x H for 0.5B and 7B)
             ("allreduce", 2048, 896), ("allreduce", 2048, 3584)]
# kr_qwen_profile_many op -> reference cost-table key (shapes of the model's config)
QWEN_KEYS = {
    "matmul_q": lambda c, S: "matmul|%dx%dx%d" % (S, c["H"], c["HQ"] * c["D"]),
    "matmul_k": lambda c, S: "matmul|%dx%dx%d" % (S, c["H"], c["HKV"] * c["D"]),
    "matmul_o": lambda c, S: "matmul|%dx%dx%d" % (S, c["HQ"] * c["D"], c["H"]),
    "matmul_gate": lambda c, S: "matmul|%dx%dx%d" % (S, c["H"], c["I"]),
    "matmul_down": lambda c, S: "matmul|%dx%dx%d" % (S, c["I"], c["H"]),
    "matmul_lm": lambda c, S: "matmul|%dx%dx%d" % (S, c["H"], c["V"]),
    "attention": lambda c, S: "attention|1x%dx%dx%d" % (c["HQ"], S, c["D"]),
    "rmsnorm": lambda c, S: "rmsnorm|%dx%d" % (S, c["H"]),
    "add_rmsnorm": lambda c, S: "add_rmsnorm|%dx%d" % (S, c["H"]),
    "rope": lambda c, S: "rope|%dx%d" % (S, c["HQ"] * c["D"]),
    "add": lambda c, S: "add|%dx%d" % (S, c["H"]),
    "silu": lambda c, S: "silu|%dx%d" % (S, c["I"]),
    "mul": lambda c, S: "mul|%dx%d" % (S, c["I"]),
    "embedding": lambda c, S: "embedding|%dx%d" % (S, c["H"]),
}


def node_of(name, op, shape):
    """Executor node fields of a DAG shape (scheduler/export.py node_dims)."""
    if op == "matmul":
        return {"id": name, "op": op, "rows": shape["M"], "cols": shape["N"], "k": shape["K"],
                "n": shape["N"]}
    n = {"id": name, "op": op, "rows": shape["rows"], "cols": shape["cols"]}
    if op == "topk":
        n["k"] = shape["k"]
    if op == "embedding":
        n["dim0"] = shape.get("vocab", 32000)
    return n


def split_schedule(name, op, strategy, shape, k, nranks=1, engine=None):
    """One node, k tasks back to back on one lane (row or matmul column tiles)."""
    node = node_of(name, op, shape)
    node.update(engine=engine or ("aic" if op == "matmul" else "aiv"), preds=[], iters=1,
                blocks=1, dtype="fp16", tiles=k, split=k > 1)
    tasks = []
    for t in range(k):
        if strategy == "col":
            w = node["n"] // k
            tasks.append({"node": name, "tile": t, "wait": [], "publish": False, "in_row_off": 0,
                          "in_rows": node["rows"], "out_row_off": 0, "n_off": t * w,
                          "n_tiles": w if k > 1 else 0, "out_col_off": t * w,
                          "out_cols": w if k > 1 else 0})
        else:
            r = node["rows"] // k
            tasks.append({"node": name, "tile": t, "wait": [], "publish": False,
                          "in_row_off": t * r, "in_rows": r, "out_row_off": t * r})
    return {"dag": "e1_" + name, "group": "standalone_c%d" % k, "nranks": nranks,
            "nodes": [node], "streams": {node["engine"]: tasks}}


def valid_k(op, strategy, shape, k):
    if strategy == "col":
        return shape["N"] % k == 0 and (shape["N"] // k) % 8 == 0
    rows = shape["M"] if op == "matmul" else shape["rows"]
    return rows % k == 0


def best_device_us(sched, devices, iters, warmup, mode="direct"):
    with tempfile.TemporaryDirectory() as td:
        p = Path(td) / "s.json"
        p.write_text(json.dumps(sched), encoding="utf-8")
        r = libapi.plan_run(p, devices=devices, mode=mode, iters=iters, warmup=warmup,
                            out_json=Path(td) / "o.json")
    if r.get("_rc") != 0:
        raise RuntimeError("%s: %s" % (sched["dag"], r.get("error")))
    return min(r["device_times_us"])


def fit(samples, holdout_k):
    """total(k) = intercept + slope * (k - 1) by least squares; MAPE over every k; the
    holdout point is predicted from a fit without it."""
    def lsq(pts):
        n = len(pts)
        xs = [k - 1 for k, _ in pts]
        ys = [v for _, v in pts]
        mx, my = sum(xs) / n, sum(ys) / n
        sxx = sum((x - mx) ** 2 for x in xs)
        slope = sum((x - mx) * (y - my) for x, y in zip(xs, ys)) / sxx if sxx else 0.0
        return slope, my - slope * mx
    pts = sorted(samples.items())
    slope, icpt = lsq(pts)
    mape = sum(abs(icpt + slope * (k - 1) - v) / v for k, v in pts) / len(pts)
    out = {"slope_us_per_tile": slope, "intercept_us": icpt, "mape_all": mape}
    rest = [(k, v) for k, v in pts if k != holdout_k]
    if len(rest) >= 2 and holdout_k in samples:
        s2, i2 = lsq(rest)
        out["holdout_k"] = float(holdout_k)
        out["holdout_ape"] = abs(i2 + s2 * (holdout_k - 1) - samples[holdout_k]) / samples[holdout_k]
    return out


def measure_curves(devices, iters, warmup, ks=KS, log=print):
    dev0 = devices.split(",")[0]
    cases = []
    for name, op, strategy, shape in CURVE_CASES:
        samples = {}
        for k in ks:
            if not valid_k(op, strategy, shape, k):
                continue
            samples[k] = best_device_us(split_schedule(name, op, strategy, shape, k), dev0,
                                        iters, warmup)
        case = {"case": name, "op": op, "strategy": strategy, "shape": shape,
                "base_best_us": samples[1], "samples_us": {str(k): v for k, v in samples.items()},
                "fit": fit(samples, max(samples))}
        log(json.dumps({"case": name, "base_best_us": round(samples[1], 2),
                        "slope_us_per_tile": round(case["fit"]["slope_us_per_tile"], 3)}))
        cases.append(case)
    return cases


def shape_key(op, shape):
    if op == "matmul":
        return "matmul|%dx%dx%d" % (shape["M"], shape["K"], shape["N"])
    return "%s|%dx%d" % (op, shape["rows"], shape["cols"])


def measure_overheads(dev0, iters, warmup):
    """Per-launch cost (extra device time per additional tiny task on one lane) and the
    cost of one cross-stream record/wait edge (a 16-task chain alternating two lanes
    against the same chain on one lane)."""
    shape = {"rows": 256, "cols": 256}
    t1 = best_device_us(split_schedule("tiny", "gelu", "row", shape, 1), dev0, iters, warmup)
    t16 = best_device_us(split_schedule("tiny", "gelu", "row", shape, 16), dev0, iters, warmup)
    launch = max(0.0, (t16 - t1) / 15.0)
    one = split_schedule("tiny", "gelu", "row", shape, 16)
    two = json.loads(json.dumps(one))
    tasks = two["streams"].pop("aiv")
    lanes = {"aic": [], "aiv": []}
    for i, t in enumerate(tasks):
        t["publish"] = True
        if i:
            t["wait"] = [["tiny", i - 1]]
        lanes["aic" if i % 2 == 0 else "aiv"].append(t)
    two["streams"] = lanes
    for t in one["streams"]["aiv"]:
        t["publish"] = True
    ev = (best_device_us(two, dev0, iters, warmup) - best_device_us(one, dev0, iters, warmup)) / 15.0
    return launch, max(0.0, ev)


def measure_qwen(config, seq, device, log=print):
    from kernrelay_b200 import model_gen, profile_model
    cfg = model_gen.CONFIGS[config]
    c = {"H": cfg.H, "HQ": cfg.HQ, "HKV": cfg.HKV, "D": cfg.D, "I": cfg.I, "V": cfg.V}
    with tempfile.TemporaryDirectory() as td:
        mdir = model_gen.write_model(Path(td) / "m", cfg, seq, seed=1234, materialize=False)
        table = profile_model.profile(mdir, seq, device, [1])["table"]
    full = {}
    for op, keyf in QWEN_KEYS.items():
        if op in table and 1 in table[op]:
            full[keyf(c, seq)] = table[op][1]
    log(json.dumps({"qwen": config, "keys": len(full)}))
    return full


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out-dir", required=True)
    ap.add_argument("--devices", default="0")
    ap.add_argument("--qwen", default="qwen2.5-0.5b,qwen2.5-7b",
                    help="model architectures whose operator costs enter the table ('' = none)")
    ap.add_argument("--seq", type=int, default=2048)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--merge-into", help="existing cost table: re-measure only the Qwen "
                                         "operator keys into it (curves, collectives kept)")
    args = ap.parse_args()
    out = Path(args.out_dir)
    if args.merge_into:
        costs = json.loads(Path(args.merge_into).read_text(encoding="utf-8"))
        for cfg in [c for c in args.qwen.split(",") if c]:
            costs["full"].update({k: round(v, 3) for k, v in
                                  measure_qwen(cfg, args.seq, int(args.devices.split(",")[0])).items()})
        costs["full"] = dict(sorted(costs["full"].items()))
        out.mkdir(parents=True, exist_ok=True)
        dst = out / Path(args.merge_into).name
        dst.write_text(json.dumps(costs, indent=1) + "\n", encoding="utf-8")
        print(json.dumps({"out": str(dst), "full": len(costs["full"])}))
        return
    out.mkdir(parents=True, exist_ok=True)
    devs = args.devices.split(",")
    dev0 = devs[0]

    cases = measure_curves(args.devices, args.iters, args.warmup)
    full = {}
    for case in cases:
        full[shape_key(case["op"], case["shape"])] = case["base_best_us"]
    for op, shape in EXTRA_FULL:
        key = shape_key(op, shape)
        if key not in full:
            full[key] = best_device_us(split_schedule("x", op, "row", shape, 1), dev0,
                                       args.iters, args.warmup)
    comm_note = "collectives not measured (one device)"
    if len(devs) >= 2:
        n = len(devs)
        for op, rows, cols in COMM_FULL:
            sched = split_schedule("c", op, "row", {"rows": rows, "cols": cols}, 1, nranks=n,
                                   engine="hccl")
            full["%s|%dx%d" % (op, rows, cols)] = best_device_us(sched, args.devices, args.iters,
                                                                 args.warmup)
        comm_note = "collectives over %d GPUs (NCCL)" % n
    for cfg in [c for c in args.qwen.split(",") if c]:
        full.update(measure_qwen(cfg, args.seq, int(dev0)))
    launch, event = measure_overheads(dev0, args.iters, args.warmup)
    # streaming bandwidth of the plainest op: add reads two operands and writes one
    add = next(c for c in cases if c["case"] == "add_huge")
    gbps = 3 * add["shape"]["rows"] * add["shape"]["cols"] * 2 / (add["base_best_us"] * 1e-6) / 1e9
    row_slopes = sorted(c["fit"]["slope_us_per_tile"] for c in cases if c["strategy"] == "row")
    col = next(c for c in cases if c["strategy"] == "col")
    costs = {
        "description": "planner2 cost table measured on B200 by kr_plan_run / kr_qwen_profile_many "
                       "(device time, best of %d); %s" % (args.iters, comm_note),
        "launch_us": round(launch, 3),
        "traffic_gbps": round(gbps, 1),
        "l2_mb": 126.0,
        "event_us": round(event, 3),
        "full": {k: round(v, 3) for k, v in sorted(full.items())},
        "split": {
            "row": {"overhead_per_tile_us": round(row_slopes[len(row_slopes) // 2], 3),
                    "traffic_factor": 1.0,
                    "note": "median E1 row-curve slope; row tiles write contiguous outputs"},
            "col": {"overhead_per_tile_us": round(col["fit"]["slope_us_per_tile"], 3),
                    "viewcopy_per_mb_us": 0.0,
                    "note": "N tiles store straight into the strided output (no copy)"},
            "m2d": {"overhead_per_tile_us": round(col["fit"]["slope_us_per_tile"], 3),
                    "viewcopy_per_mb_us": 0.0, "note": "as col"},
        },
    }
    curves = {"description": "E1 split curves measured on B200 through kr_plan_run (k tasks back "
                             "to back on one lane, best device time): total time of k "
                             "consecutive tiles", "cases": cases}
    (out / "planner2_costs_b200.json").write_text(json.dumps(costs, indent=1) + "\n", encoding="utf-8")
    (out / "planner_curves_b200.json").write_text(json.dumps(curves, indent=1) + "\n", encoding="utf-8")
    print(json.dumps({"out": str(out), "cases": len(cases), "full": len(full),
                      "launch_us": costs["launch_us"], "event_us": costs["event_us"],
                      "traffic_gbps": costs["traffic_gbps"]}))


if __name__ == "__main__":
    main()
