"""kr_plan_run: the generic schedule executor (reference exec/exec_main.cpp RunPlanCli).

Schedules are the reference scheduler's own output (tests/golden/plans, made by
tests/golden/make_plan_schedules.py).  CPU tests cover parsing, validation and the
reference's rejection variants through the C ABI, and properties of the CPU oracle;
GPU tests compare the CUDA executor's per-node checksums with the oracle
(oracle/plan_ref.py) for every small schedule and every launch mode.
"""
import copy
import json
from pathlib import Path

import numpy as np
import pytest

from oracle import plan_ref

PLANS = Path(__file__).resolve().parent / "golden" / "plans"
MANIFEST = json.loads((PLANS / "manifest.json").read_text(encoding="utf-8"))
SMALL = [e for e in MANIFEST["schedules"] if e["size"] == "small"]
FULL = [e for e in MANIFEST["schedules"] if e["size"] == "full"]
MODES = ("direct", "graph", "graph_per_stream", "graph_segment")

# per-node checksum tolerance: one fp16 rounding (2^-11 relative) per element of the
# 8192 summed, against the oracle's sum of |values|
REL_TOL = 1e-3


def _load(entry):
    return json.loads((PLANS / entry["file"]).read_text(encoding="utf-8"))


def _ids(entries):
    return [e["file"] for e in entries]


# ---------------------------------------------------------------- CPU: boundary + oracle
@pytest.mark.parametrize("entry", SMALL + FULL, ids=_ids(SMALL + FULL))
def test_plan_check_accepts_reference_schedules(krlib, entry):
    sched = _load(entry)
    info = krlib.plan_check(PLANS / entry["file"])
    assert info["dag"] == sched["dag"] and info["nranks"] == sched["nranks"]
    assert info["nodes"] == len(sched["nodes"])
    assert info["tasks"] == sum(len(v) for v in sched["streams"].values())
    assert info["publishes"] == sum(bool(t.get("publish")) for v in sched["streams"].values()
                                    for t in v)


@pytest.mark.parametrize("entry", MANIFEST["invalid"], ids=[e["variant"] for e in MANIFEST["invalid"]])
def test_rejection_variants(krlib, entry, tmp_path):
    """schedule.py invalid_variants: each mutation fails with the reference's message,
    through krb_plan_check and through kr_plan_run (before any device work)."""
    from kernrelay_b200 import libapi
    with pytest.raises(krlib.KrbError, match=entry["expect"]):
        krlib.plan_check(PLANS / entry["file"])
    r = libapi.plan_run(PLANS / entry["file"], devices="", mode="direct",
                        out_json=tmp_path / "o.json")
    assert r["_rc"] == 1 and entry["expect"] in r["error"]


def test_plan_run_argument_errors(krlib, tmp_path):
    from kernrelay_b200 import libapi
    s = PLANS / "small" / "f03_mm_ar_c4_b.json"   # nranks 2
    r = libapi.plan_run(s, devices="0", mode="direct", out_json=tmp_path / "a.json")
    assert r["_rc"] == 1 and "devices needs exactly 2 devices" in r["error"]
    r = libapi.plan_run(s, devices="0,", mode="direct", out_json=tmp_path / "b.json")
    assert r["_rc"] == 1 and "empty entry" in r["error"]
    r = libapi.plan_run(s, devices="0,1", mode="bogus", out_json=tmp_path / "c.json")
    assert r["_rc"] == 1 and "unknown plan mode" in r["error"]
    bad = _load({"file": "small/e0_tiny_mm_gelu_b.json"})
    bad["nodes"][0]["op"] = "conv"
    p = tmp_path / "bad_op.json"
    p.write_text(json.dumps(bad))
    with pytest.raises(krlib.KrbError, match="unknown op: conv"):
        krlib.plan_check(p)
    bad = _load({"file": "small/e0_tiny_mm_gelu_b.json"})
    bad["streams"]["tpu"] = []
    p.write_text(json.dumps(bad))
    with pytest.raises(krlib.KrbError, match="unknown engine tpu"):
        krlib.plan_check(p)


def test_graph_per_stream_needs_acyclic_lanes(krlib):
    """e9_chain2 (mm1 -> gelu1 -> mm2 -> gelu2 on aic/aiv) ping-pongs between two lanes,
    so one graph per lane cannot order it; the executor says so up front."""
    info = krlib.plan_check(PLANS / "small" / "e9_chain2_b.json")
    assert info["lane_order_acyclic"] is False
    assert krlib.plan_check(PLANS / "small" / "f02_mm_gelu_c4_b.json")["lane_order_acyclic"]


def test_oracle_inputs_follow_detvalue():
    v = plan_ref.det_values(12345, 4096)
    k = np.round(v * 256).astype(np.int64)
    assert np.allclose(k / 256.0, v) and k.min() >= -11 and k.max() <= 11
    assert len(np.unique(k)) == 23
    # index truncation to 32 bits (exec_main.cpp:76 casts index to uint32)
    big = plan_ref.det_values(7, 0, index=[5, (1 << 32) + 5])
    assert big[0] == big[1]
    assert plan_ref.node_seed("mm", 1) == (plan_ref.node_seed("mm", 0) + 7919) & 0xFFFFFFFF


@pytest.mark.parametrize("dag", sorted({e["dag"] for e in SMALL}))
def test_oracle_tiling_invariance(dag):
    """A-nosplit, B-split and serial schedules of one DAG compute the same outputs, except
    the scalar accumulation probes, whose accumulator runs over one task's elements."""
    entries = [e for e in SMALL if e["dag"] == dag]
    runs = {e["group"]: plan_ref.run_file(PLANS / e["file"]) for e in entries}
    ops = {n["id"]: n["op"] for n in _load(entries[0])["nodes"]}
    base = runs["a"]["node_checksums"]
    for g, r in runs.items():
        for nid, v in r["node_checksums"].items():
            if ops[nid] in ("custom_aic_mac", "custom_aicpu_scale"):
                continue
            assert v == pytest.approx(base[nid], rel=0, abs=1e-9), (g, nid)


def test_oracle_matmul_gelu_against_torch():
    """mm -> gelu of the tiny E0 DAG recomputed with torch from the same inputs."""
    import torch
    sched = _load({"file": "small/e0_tiny_mm_gelu_a.json"})
    mm = next(n for n in sched["nodes"] if n["op"] == "matmul")
    seed = plan_ref.node_seed(mm["id"], 0)
    A = torch.tensor(plan_ref.det_values(seed + 1, mm["rows"] * mm["k"])).reshape(mm["rows"], mm["k"])
    B = torch.tensor(plan_ref.det_values(seed + 2, mm["k"] * mm["n"])).reshape(mm["k"], mm["n"])
    C = (A.double() @ B.double()).float().half()
    G = torch.nn.functional.gelu(C.float(), approximate="tanh").half()
    r = plan_ref.run_file(PLANS / "small" / "e0_tiny_mm_gelu_a.json")
    assert r["node_checksums"]["mm"] == pytest.approx(C.flatten()[:8192].double().sum().item(), abs=1e-6)
    gsum = G.flatten()[:8192].double().sum().item()
    assert r["node_checksums"]["gelu"] == pytest.approx(gsum, abs=1e-3 * G.abs().double().sum().item())


# ---------------------------------------------------------------- GPU parity
def _one_rank(sched):
    """The schedule with nranks 1 (collectives become single-rank NCCL calls), so every
    DAG runs on one GPU."""
    s = copy.deepcopy(sched)
    s["nranks"] = 1
    return s


def _compare(res, ref, what):
    assert res["_rc"] == 0, res
    assert res["ok"] and res["device_status"] == 0, res
    for nid, v in ref["node_checksums"].items():
        tol = REL_TOL * ref["node_abs"][nid] + 1e-6
        assert abs(res["node_checksums"][nid] - v) <= tol, (what, nid, res["node_checksums"][nid], v)


@pytest.mark.gpu
@pytest.mark.parametrize("entry", SMALL, ids=_ids(SMALL))
def test_plan_parity_direct(krlib, cuda, entry, tmp_path):
    from kernrelay_b200 import libapi
    sched = _one_rank(_load(entry))
    p = tmp_path / "s.json"
    p.write_text(json.dumps(sched))
    ref = plan_ref.PlanOracle(sched).run()
    res = libapi.plan_run(p, devices="0", mode="direct", iters=2, warmup=1,
                          out_json=tmp_path / "o.json")
    _compare(res, ref, entry["file"])
    assert len(res["times_us"]) == 2 and res["device_p50_us"] > 0


@pytest.mark.gpu
@pytest.mark.parametrize("mode", MODES[1:])
@pytest.mark.parametrize("name", ["f02_mm_gelu_c4_b", "e9_mixed_b", "e4_mm_cross_aicpu_b",
                                  "e3_ln_mm_b", "e5_mm_ag_part_b", "e9_chain2_b"])
def test_plan_parity_graph_modes(krlib, cuda, name, mode, tmp_path):
    from kernrelay_b200 import libapi
    sched = _one_rank(_load({"file": f"small/{name}.json"}))
    p = tmp_path / "s.json"
    p.write_text(json.dumps(sched))
    res = libapi.plan_run(p, devices="0", mode=mode, iters=3, warmup=1, out_json=tmp_path / "o.json")
    if mode == "graph_per_stream" and name == "e9_chain2_b":
        assert res["_rc"] == 1 and "acyclic" in res["error"]
        return
    _compare(res, plan_ref.PlanOracle(sched).run(), f"{name}/{mode}")


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["f02_mm_gelu_c4", "e3_mm_softmax", "e9_two_waves"])
def test_plan_full_size_tiling_invariance(krlib, cuda, name, tmp_path):
    """Full DAG shapes (M = 32768): the split schedule in graph mode reproduces the
    oracle's checksum of the first 8192 outputs, computed on the rows that feed them."""
    from kernrelay_b200 import libapi
    sched = _load({"file": f"full/{name}_b.json"})
    res = libapi.plan_run(PLANS / "full" / f"{name}_b.json", devices="0", mode="graph", iters=2,
                          warmup=1, out_json=tmp_path / "o.json")
    assert res["_rc"] == 0 and res["ok"], res
    # every node of these DAGs is row-wise, so the first 8192 outputs depend only on the
    # first rows: run the oracle on a row-truncated copy of the same schedule
    small = copy.deepcopy(sched)
    keep = 64
    for n in small["nodes"]:
        n["rows"] = keep
        n["tiles"] = 1
        n["split"] = False
    for lane in small["streams"].values():
        lane[:] = [t for t in lane if int(t.get("tile", 0)) == 0]
        for t in lane:
            t["in_row_off"], t["in_rows"], t["out_row_off"] = 0, keep, 0
            t["wait"] = [w for w in t.get("wait") or [] if int(w[1]) == 0]
    ref = plan_ref.PlanOracle(small).run()
    _compare(res, ref, name)


@pytest.mark.gpu
@pytest.mark.multigpu
@pytest.mark.parametrize("name", ["f03_mm_ar_c4_b", "e5_mm_ag_part_b", "e5_mm_rs_part_b",
                                  "e4_mm_cross_hccl_b", "e5_mm_ar_full_b"])
def test_plan_parity_two_ranks(krlib, cuda, name, tmp_path):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from kernrelay_b200 import libapi
    sched = _load({"file": f"small/{name}.json"})
    assert sched["nranks"] == 2
    ref = plan_ref.PlanOracle(sched).run()
    for mode in ("direct", "graph"):
        res = libapi.plan_run(PLANS / "small" / f"{name}.json", devices="0,1", mode=mode, iters=2,
                              warmup=1, out_json=tmp_path / f"{mode}.json")
        _compare(res, ref, f"{name}/{mode}")


# ---------------------------------------------------------------- every operator kind
def _standalone(name, node, chunks=1, engine="aiv", col_tiles=0):
    """A one-node schedule in the scheduler's standalone form (schedule.py:57-64): the node
    split into `chunks` row tasks (or `col_tiles` matmul N tiles) on one engine lane."""
    n = dict(node, id=name, engine=engine, preds=[], iters=node.get("iters", 1),
             blocks=node.get("blocks", 1), dtype="fp16")
    tasks = []
    if col_tiles:
        n.update(tiles=col_tiles, split=True)
        w = n["n"] // col_tiles
        for t in range(col_tiles):
            tasks.append({"node": name, "tile": t, "wait": [], "publish": False,
                          "in_row_off": 0, "in_rows": n["rows"], "out_row_off": 0,
                          "n_off": t * w, "n_tiles": w, "out_col_off": t * w, "out_cols": w})
    else:
        n.update(tiles=chunks, split=chunks > 1)
        r = n["rows"] // chunks
        for t in range(chunks):
            tasks.append({"node": name, "tile": t, "wait": [], "publish": False,
                          "in_row_off": t * r, "in_rows": r, "out_row_off": t * r})
    return {"dag": "ops_" + name, "group": "standalone", "nranks": 1, "nodes": [n],
            "streams": {engine: tasks}}


OP_CASES = {
    "add": ({"op": "add", "rows": 256, "cols": 512}, 2),
    "gelu_ragged": ({"op": "gelu", "rows": 100, "cols": 333}, 1),
    "softmax_long": ({"op": "softmax", "rows": 64, "cols": 5000}, 1),
    "softmax_warp": ({"op": "softmax", "rows": 128, "cols": 1000}, 2),
    "layernorm_ragged": ({"op": "layernorm", "rows": 64, "cols": 300}, 1),
    "layernorm_wide": ({"op": "layernorm", "rows": 96, "cols": 4096}, 3),
    "cast": ({"op": "cast", "rows": 128, "cols": 256}, 2),
    "topk": ({"op": "topk", "rows": 64, "cols": 1000, "k": 16}, 2),
    "sort": ({"op": "sort", "rows": 32, "cols": 700}, 1),
    "embedding": ({"op": "embedding", "rows": 128, "cols": 256, "dim0": 1000}, 2),
    "aiv_scale": ({"op": "custom_aiv_scale", "rows": 64, "cols": 512, "iters": 3}, 1),
    "mix_scale": ({"op": "custom_mix_scale", "rows": 64, "cols": 512, "iters": 2}, 2),
    "aic_mac": ({"op": "custom_aic_mac", "rows": 64, "cols": 512, "iters": 2, "blocks": 4}, 2),
    "aicpu_scale": ({"op": "custom_aicpu_scale", "rows": 64, "cols": 256}, 1),
}


def _op_schedule(name):
    if name == "matmul_ntiles":
        return _standalone(name, {"op": "matmul", "rows": 256, "cols": 512, "k": 128, "n": 512},
                           engine="aic", col_tiles=2)
    node, chunks = OP_CASES[name]
    return _standalone(name, node, chunks)


OP_NAMES = sorted(OP_CASES) + ["matmul_ntiles"]


@pytest.mark.parametrize("name", OP_NAMES)
def test_op_schedules_validate_and_run_on_oracle(krlib, name, tmp_path):
    sched = _op_schedule(name)
    p = tmp_path / "s.json"
    p.write_text(json.dumps(sched))
    assert krlib.plan_check(p)["tasks"] == len(next(iter(sched["streams"].values())))
    r = plan_ref.PlanOracle(sched).run()
    assert np.isfinite(r["checksum"]) and r["node_abs"][name] > 0


def test_oracle_topk_sort_semantics():
    sched = _op_schedule("topk")
    o = plan_ref.PlanOracle(sched)
    o.run()
    node = sched["nodes"][0]
    seed = plan_ref.node_seed("topk", 0)
    x = plan_ref.det_values(seed + 1, node["rows"] * node["cols"]).reshape(node["rows"], node["cols"])
    vals = o.buf[0]["topk"]["out"].view(np.float16)[:node["rows"] * 16].reshape(node["rows"], 16)
    idx = o.buf[0]["topk"]["out2"].reshape(node["rows"], 16)
    assert np.array_equal(vals.astype(np.float32), -np.sort(-x, axis=1)[:, :16])
    assert np.array_equal(np.take_along_axis(x, idx, axis=1), vals.astype(np.float32))
    # ties (23 distinct values) resolve to the lower index first
    for r in range(node["rows"]):
        for j in range(15):
            if vals[r, j] == vals[r, j + 1]:
                assert idx[r, j] < idx[r, j + 1]


@pytest.mark.gpu
@pytest.mark.parametrize("name", OP_NAMES)
def test_op_schedules_gpu_parity(krlib, cuda, name, tmp_path):
    from kernrelay_b200 import libapi
    sched = _op_schedule(name)
    p = tmp_path / "s.json"
    p.write_text(json.dumps(sched))
    ref = plan_ref.PlanOracle(sched).run()
    for mode in ("direct", "graph"):
        res = libapi.plan_run(p, devices="0", mode=mode, iters=2, warmup=1,
                              out_json=tmp_path / f"{mode}.json")
        _compare(res, ref, f"{name}/{mode}")


# ---------------------------------------------------------------- planner cost tables (row f3)
def test_planner_curve_schedules_validate(krlib, tmp_path):
    from kernrelay_b200 import planner_costs as pc
    n = 0
    for name, op, strategy, shape in pc.CURVE_CASES:
        ks = [k for k in pc.KS if pc.valid_k(op, strategy, shape, k)]
        assert 1 in ks and len(ks) >= 4, name
        for k in ks:
            s = pc.split_schedule(name, op, strategy, shape, k)
            p = tmp_path / f"{name}_{k}.json"
            p.write_text(json.dumps(s))
            assert krlib.plan_check(p)["tasks"] == k
            n += 1
    assert n > 80


def test_planner_fit_recovers_linear_total():
    from kernrelay_b200 import planner_costs as pc
    samples = {k: 250.0 + 7.5 * (k - 1) for k in (1, 2, 4, 8, 16)}
    f = pc.fit(samples, 16)
    assert f["slope_us_per_tile"] == pytest.approx(7.5)
    assert f["intercept_us"] == pytest.approx(250.0)
    assert f["mape_all"] < 1e-12 and f["holdout_ape"] < 1e-12


# ---------------------------------------------------------------- oracle vs torch operators
def _torch_eval(sched):
    """Independent evaluation of an unsplit (one task per node) schedule with PyTorch's own
    operators -- the semantics CANN's aclnn ops follow -- rounding to fp16 where the
    executor stores fp16: matmul (fp32 accumulate), tanh-GELU, softmax, layer_norm (eps
    1e-5), cast, stable topk / sort, embedding, add, the custom scale ops, and the
    collectives as sums / concatenations over ranks.  Returns node -> checksum."""
    import torch
    R = int(sched.get("nranks", 1))
    nodes = {n["id"]: n for n in sched["nodes"]}
    order = [t["node"] for lane in sorted(sched["streams"]) for t in sched["streams"][lane]]
    # topological order of nodes (every node of an A schedule has one task)
    done, topo = set(), []
    while len(topo) < len(nodes):
        for nid in order:
            if nid not in done and all(p in done for p in nodes[nid].get("preds", [])):
                done.add(nid)
                topo.append(nid)
    f16 = lambda x: x.to(torch.float16).to(torch.float32)  # noqa: E731
    out = [{} for _ in range(R)]
    sums = {}
    for nid in topo:
        n = nodes[nid]
        op, rows, cols = n["op"], int(n["rows"]), int(n.get("cols", 0))
        for r in range(R):
            seed = plan_ref.node_seed(nid, r)
            in_cols = int(n["k"]) if op == "matmul" else cols
            if n.get("preds"):
                x = out[r][n["preds"][0]][:rows * in_cols].reshape(rows, in_cols)
            elif op != "embedding":
                x = f16(torch.tensor(plan_ref.det_values(seed + 1, rows * in_cols))).reshape(rows, in_cols)
            if op == "matmul":
                B = f16(torch.tensor(plan_ref.det_values(seed + 2, int(n["k"]) * int(n["n"])))).reshape(int(n["k"]), -1)
                y = f16((x.double() @ B.double()).float())
            elif op == "gelu":
                y = f16(torch.nn.functional.gelu(x, approximate="tanh"))
            elif op == "softmax":
                y = f16(torch.softmax(x, dim=-1))
            elif op == "layernorm":
                w = f16(torch.tensor(plan_ref.det_values(seed + 2, cols)))
                b = f16(torch.tensor(plan_ref.det_values(seed + 3, cols)))
                y = f16(torch.nn.functional.layer_norm(x, (cols,), w, b, eps=1e-5))
            elif op == "cast":
                y = x.clone()
            elif op in ("custom_aiv_scale", "custom_mix_scale"):
                k = 1.0009765625 if op == "custom_aiv_scale" else 1.001953125
                y = f16(x * k)
            elif op == "add":
                other = (out[r][n["preds"][1]][:rows * cols].reshape(rows, cols)
                         if len(n.get("preds", [])) > 1 else
                         f16(torch.tensor(plan_ref.det_values(seed + 3, rows * cols))).reshape(rows, cols))
                y = f16(x + other)
            elif op == "topk":
                v = torch.topk(x, int(n["k"]), dim=-1, largest=True, sorted=True).values
                y = torch.cat([v.flatten(), torch.zeros(rows * int(n["k"]) * 4)])  # index bytes follow
            elif op == "sort":
                v = torch.sort(x, dim=-1, stable=True).values
                y = torch.cat([v.flatten(), torch.zeros(rows * cols * 4)])
            elif op == "embedding":
                V = int(n["dim0"])
                W = f16(torch.tensor(plan_ref.det_values(seed + 2, V * cols))).reshape(V, cols)
                i = torch.arange(rows, dtype=torch.int64)
                y = W[(i * 131 + 7 + seed) % V]
            else:
                y = None  # collectives below; the DAGs' other ops are covered above
            if y is not None:
                out[r][nid] = y.flatten()
        if op in ("allreduce", "reducescatter", "allgather"):
            xs = [out[r][n["preds"][0]][:rows * cols] if n.get("preds") else
                  f16(torch.tensor(plan_ref.det_values(plan_ref.node_seed(nid, r) + 1, rows * cols)))
                  for r in range(R)]
            if op == "allreduce":
                s = xs[0]
                for x in xs[1:]:
                    s = f16(s + x)
                for r in range(R):
                    out[r][nid] = s
            elif op == "reducescatter":
                s = xs[0]
                for x in xs[1:]:
                    s = f16(s + x)
                cnt = rows * cols // R
                for r in range(R):
                    buf = torch.zeros(rows * cols)
                    lo = (r * rows // R) * cols
                    buf[lo:lo + cnt] = s[r * cnt:(r + 1) * cnt]
                    out[r][nid] = buf
            else:
                cat = torch.cat(xs)
                for r in range(R):
                    out[r][nid] = cat
        if nid in out[0]:
            sums[nid] = sum(float(out[r][nid][:8192].double().sum()) for r in range(R))
    return sums


@pytest.mark.parametrize("entry", [e for e in SMALL if e["group"] == "a"], ids=lambda e: e["dag"])
def test_oracle_matches_torch_operators(entry):
    """Pin of the executor oracle: every reference DAG (unsplit schedule, small shapes)
    evaluated independently with PyTorch's operators gives the oracle's node checksums.
    The scalar accumulation probes are left to the oracle's own restatement."""
    sched = _load(entry)
    ref = plan_ref.PlanOracle(sched).run()
    got = _torch_eval(sched)
    checked = 0
    for nid, v in got.items():
        tol = REL_TOL * ref["node_abs"][nid] + 1e-6
        assert abs(v - ref["node_checksums"][nid]) <= tol, (entry["dag"], nid, v, ref["node_checksums"][nid])
        checked += 1
    assert checked >= 1


@pytest.mark.parametrize("name", [n for n in OP_NAMES if n not in ("aic_mac", "aicpu_scale")])
def test_op_schedules_oracle_matches_torch_operators(name):
    """The same pin for the operator kinds no reference DAG uses (add, topk, sort,
    embedding, ragged shapes, matmul N tiles): row-wise ops, so the schedule's chunking does
    not change the checksum."""
    sched = _op_schedule(name)
    ref = plan_ref.PlanOracle(sched).run()
    got = _torch_eval(sched)
    assert name in got
    tol = REL_TOL * ref["node_abs"][name] + 1e-6
    assert abs(got[name] - ref["node_checksums"][name]) <= tol, (name, got[name], ref["node_checksums"][name])


@pytest.mark.parametrize("name", ["e5_mm_ar_full_a", "e5_mm_ag_part_a", "e5_mm_rs_part_a",
                                  "f03_mm_ar_c4_a", "e4_mm_cross_hccl_a", "e9_mixed_a"])
def test_collective_dags_at_four_ranks_match_torch(name):
    """The collective DAGs with nranks = 4: reduce-scatter blocks at rank * rows / 4,
    all-gather placement by rank, allreduce sums -- oracle against the torch evaluation."""
    sched = _load({"file": f"small/{name}.json"})
    sched["nranks"] = 4
    ref = plan_ref.PlanOracle(sched).run()
    got = _torch_eval(sched)
    for nid, v in got.items():
        tol = REL_TOL * ref["node_abs"][nid] + 1e-6
        assert abs(v - ref["node_checksums"][nid]) <= tol, (name, nid, v, ref["node_checksums"][nid])


def test_committed_planner_tables_keep_the_reference_format():
    """kernrelay_b200/configs/*_b200.json are read by the reference planner's Costs class
    (launch_us, traffic_gbps, l2_mb, event_us, full; curve cases keyed by op and shape with
    base_best_us and fit.slope_us_per_tile / fit.intercept_us)."""
    cfg = Path(__file__).resolve().parents[1] / "kernrelay_b200" / "configs"
    costs = json.loads((cfg / "planner2_costs_b200.json").read_text(encoding="utf-8"))
    curves = json.loads((cfg / "planner_curves_b200.json").read_text(encoding="utf-8"))
    for key in ("launch_us", "traffic_gbps", "l2_mb", "event_us", "full", "split"):
        assert key in costs, key
    assert all(isinstance(v, (int, float)) and v >= 0 for v in costs["full"].values())
    for op in ("matmul", "gelu", "softmax", "layernorm", "attention", "allreduce"):
        assert any(k.startswith(op + "|") for k in costs["full"]), op
    assert len(curves["cases"]) == 16
    for c in curves["cases"]:
        s = c["shape"]
        key = ("matmul|%dx%dx%d" % (s["M"], s["K"], s["N"]) if c["op"] == "matmul"
               else "%s|%dx%d" % (c["op"], s["rows"], s["cols"]))
        assert key in costs["full"], key                    # every curve's k = 1 point is a cost
        assert c["base_best_us"] > 0 and c["strategy"] in ("row", "col")
        assert c["fit"]["slope_us_per_tile"] >= 0 and c["fit"]["intercept_us"] > 0
