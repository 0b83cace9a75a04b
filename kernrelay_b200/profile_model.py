"""Per-operator k-table for the planner, measured on this GPU (the B200 counterpart of
the reference's scripts/profile_model.py): every op of the Qwen prefill at k = 1/2/4/8
row slices (head groups for attention), timed by kr_qwen_profile_many.

    python -m kernrelay_b200.profile_model --config qwen2.5-7b --seq 2048 --out table.json
    python -m kernrelay_b200.profile_model --model /path/to/model_dir --out table.json

Output JSON: {"table": {op: {k: best_us}}, "raw": <kr_qwen_profile_many result>}.
"""
import argparse
import json
import tempfile
from pathlib import Path

from kernrelay_b200 import libapi, model_gen

# the reference's operator list (scripts/profile_model.py:13-15)
OPS = ("embedding", "rmsnorm", "add", "add_rmsnorm", "rope", "matmul_q",
       "matmul_k", "matmul_v", "attention", "matmul_o", "matmul_gate",
       "matmul_up", "silu", "mul", "matmul_down", "matmul_lm")


def profile(model_dir, seq, device, ks):
    cases = [{"op": op, "k": k} for op in OPS for k in ks]
    raw = libapi.qwen_profile_many(model_dir, cases, seq=seq, device=device)
    if raw.get("_rc", 0) != 0:
        raise RuntimeError(raw.get("error", "kr_qwen_profile_many failed"))
    table = {}
    for c in raw.get("cases", []):
        if "best_us" not in c or "k" not in c:
            continue
        table.setdefault(c["op"], {})[int(c["k"])] = float(c["best_us"])
    return {"table": table, "raw": raw}


def main():
    ap = argparse.ArgumentParser()
    src = ap.add_mutually_exclusive_group(required=True)
    src.add_argument("--model", help="model directory (reference exporter layout)")
    src.add_argument("--config", help="random-init model of a named architecture "
                                      f"({', '.join(sorted(model_gen.CONFIGS))})")
    ap.add_argument("--seq", type=int, default=2048)
    ap.add_argument("--device", type=int, default=0)
    ap.add_argument("--ks", default="1,2,4,8")
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--out", required=True)
    args = ap.parse_args()
    ks = [int(x) for x in args.ks.split(",")]
    with tempfile.TemporaryDirectory() as td:
        if args.model:
            mdir = Path(args.model)
        else:
            cfg = model_gen.CONFIGS[args.config]
            mdir = model_gen.write_model(Path(td) / "m", cfg, args.seq, seed=args.seed,
                                         materialize=False)
        res = profile(mdir, args.seq, args.device, ks)
    out = Path(args.out)
    out.parent.mkdir(parents=True, exist_ok=True)
    out.write_text(json.dumps(res, indent=1), encoding="utf-8")
    print("profile", args.model or args.config, "ops", len(res["table"]), "->", out)


if __name__ == "__main__":
    main()
