"""Generate the schedule.json fixtures of the plan executor with the reference's own scheduler.

kr_plan_run consumes the schedules that the reference's Python scheduler emits
(python/kernrelay/schedule.py build_ab / serial_schedule over the DAGs in dags/).  This
script imports that scheduler from a KernRelay checkout and writes, for every DAG:

  small/<dag>_{a,b,serial}.json   shapes scaled down (rows / M by 64 from 2048 up,
                                  K, N, cols by 8 from 1024 up) for parity against the
                                  CPU oracle (oracle/plan_ref.py); same nodes, edges,
                                  engines, tiles and chunking as the DAG
  full/<dag>_{a,b}.json           the DAG's own shapes, unsplit and split
  invalid/<variant>.json          the reference's E0 rejection variants
                                  (schedule.py invalid_variants) of one small schedule

plus manifest.json.  Group a = A-nosplit, b = B-split with the DAG's fixed chunking (or
every node at its declared tiles when the DAG fixes none), serial = one lane in global
topological order.  nranks is 2 for DAGs with a collective, else 1.

Run from the repository root:
    python tests/golden/make_plan_schedules.py --reference <KernRelay checkout>
"""
from __future__ import annotations

import argparse
import copy
import glob
import json
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "plans"
COMM = {"allreduce", "allgather", "reducescatter"}


def scale_shape(shape: dict) -> dict:
    s = dict(shape)
    for k in ("M", "rows"):
        if k in s and int(s[k]) >= 2048:
            s[k] = int(s[k]) // 64
    for k in ("K", "N", "cols"):
        if k in s and int(s[k]) >= 1024:
            s[k] = int(s[k]) // 8
    return s


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="KernRelay checkout (has python/kernrelay)")
    args = ap.parse_args()
    ref = Path(args.reference)
    sys.path.insert(0, str(ref / "python"))
    from kernrelay import schedule as S  # noqa: E402  (the reference's scheduler)

    manifest = {"generator": "python/kernrelay/schedule.py build_ab / serial_schedule",
                "schedules": [], "invalid": []}
    for sub in ("small", "full", "invalid"):
        (OUT / sub).mkdir(parents=True, exist_ok=True)
    for path in sorted(glob.glob(str(ref / "dags" / "*.json"))):
        name = os.path.basename(path)[:-5]
        spec, fixed = S.load_fixed(name)
        chunking = dict(fixed) if fixed else {n.name: int(n.tiles) for n in spec.nodes
                                               if int(n.tiles) > 1}
        nranks = 2 if any(n.op in COMM for n in spec.nodes) else 1
        small = copy.deepcopy(spec)
        for n in small.nodes:
            n.shape = scale_shape(n.shape)
        for size, sp, groups in (("small", small, ("a", "b", "serial")), ("full", spec, ("a", "b"))):
            ab = S.build_ab(sp, chunking, nranks=nranks)
            built = {"a": ab["a"], "b": ab["b"], "serial": S.serial_schedule(sp, nranks=nranks)}
            for g in groups:
                sched = built[g]
                errs = S.validate_schedule(sched)
                if errs:
                    raise SystemExit(f"{name}/{g}: reference validator rejects: {errs}")
                rel = f"{size}/{name}_{g}.json"
                (OUT / rel).write_text(json.dumps(sched, indent=1, ensure_ascii=False) + "\n",
                                       encoding="utf-8")
                manifest["schedules"].append({"file": rel, "dag": name, "group": g,
                                              "size": size, "nranks": nranks,
                                              "chunking": chunking if g == "b" else {}})
    base = json.loads((OUT / "small" / "f02_mm_gelu_c4_b.json").read_text(encoding="utf-8"))
    for variant, (sched, expect) in S.invalid_variants(base).items():
        rel = f"invalid/{variant}.json"
        (OUT / rel).write_text(json.dumps(sched, indent=1, ensure_ascii=False) + "\n",
                               encoding="utf-8")
        manifest["invalid"].append({"file": rel, "variant": variant, "expect": expect})
    (OUT / "manifest.json").write_text(json.dumps(manifest, indent=1) + "\n", encoding="utf-8")
    print(f"{len(manifest['schedules'])} schedules, {len(manifest['invalid'])} invalid variants")


if __name__ == "__main__":
    main()
