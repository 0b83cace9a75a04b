"""Phase trace of the fused relay kernel: per row tile, when its partials arrived, when the
exchange and the Add+RMSNorm finished, and the NVLink bytes per second that implies.

    python -m kernrelay_b200.relay_trace --k 2 --layers 4
    python -m kernrelay_b200.relay_trace --k 4 --relay rsag --out trace.json

Runs a tp{k}_split prefill of a random-init model (all k ranks as threads of this process,
devices 0..k-1) with KRB_RELAY_TRACE=1, so every relay CTA stamps %globaltimer at its phase
boundaries (slot meanings in csrc/relay.cuh, kTraceSlots).  The last layer's relay launch is
reported, times relative to the earliest CTA start on that rank (medians over CTAs, the
latest CTA in brackets), with the signal jobs that forward each tile's completion to the
peers (when the local completion counter filled; the system-scope fence and k remote adds):

* direct (each rank pulls every peer's partial rows of tile t): NVLink bytes per rank per
  tile = (k-1) * R * H * 2, over the interval from "partials arrived" to "norm done";
* rsag (reduce-scatter then all-gather of reduced rows): the reduce-scatter pulls
  (k-1) * R/k * H * 2 bytes ("partials arrived" -> "reduced rows stored"), the all-gather
  pulls the same amount ("reduced rows arrived" -> "norm done").
A rank cannot see its peers' clocks, so these are one rank's view of its own pulls.
"""
import argparse
import json
import os
import tempfile
import threading
from pathlib import Path

import numpy as np


def run(k, layers, relay, config, seq, tiles, iters):
    os.environ["KRB_RELAY_TRACE"] = "1"
    if relay:
        os.environ["KRB_RELAY"] = relay
    from kernrelay_b200 import _lib as K, model_gen
    cfg = model_gen.config_with(config, L=layers)
    with tempfile.TemporaryDirectory() as td:
        d = model_gen.write_model(Path(td) / "m", cfg, seq, materialize=False)
        engs = [K.Engine(d, f"tp{k}_split", seq, rank=r, world=k, device=r, tiles=tiles)
                for r in range(k)]
        if k > 1:
            K.Engine.link(engs)

        def run_all():
            ts = [threading.Thread(target=lambda e=e: (e.run(), e.sync())) for e in engs]
            for t in ts:
                t.start()
            for t in ts:
                t.join()

        for _ in range(iters):
            run_all()
        traces = [e.relay_trace() for e in engs]
        status = [e.status() for e in engs]
        kind = engs[0].info().get("relay", relay or "")
        stages = engs[0].stage_times()
    return traces, status, kind, stages, cfg


def summarise(tr, k, T, R, H, kind):
    t = tr.astype(np.int64)
    t0 = t[:, 0][t[:, 0] > 0].min()

    def med(c):
        v = t[:, c]
        v = v[v > 0]
        return float(np.median(v - t0) / 1e3) if v.size else None

    def mx(c):
        v = t[:, c]
        v = v[v > 0]
        return float((v.max() - t0) / 1e3) if v.size else None

    out = {"t0_ns": int(t0), "gemm_done_us": med(1), "gemm_done_max_us": mx(1),
           "relay_end_us": med(2), "relay_end_max_us": mx(2), "tiles": [], "signals": []}
    # signal jobs (CTA j < T forwards the partials of row tile j, T <= j < 2T the reduced
    # rows of tile j - T): when the local counter completed, and the fence + remote adds
    for j in range(min(2 * T, t.shape[0])):
        end, fence = int(t[j, 46]), int(t[j, 47])
        if end > 0:
            out["signals"].append({"job": j, "tile": j % T, "kind": "ag" if j >= T else "rs",
                                   "local_done_us": (end - fence - t0) / 1e3,
                                   "forwarded_us": (end - t0) / 1e3, "fence_us": fence / 1e3})
    part_bytes = (k - 1) * R * H * 2
    slice_bytes = (k - 1) * (R // max(k, 1)) * H * 2
    for tt in range(min(T, 8)):
        arr, stored, ag, norm = med(3 + 4 * tt), med(4 + 4 * tt), med(5 + 4 * tt), med(6 + 4 * tt)
        row = {"tile": tt, "partials_arrived_us": arr, "reduced_stored_us": stored,
               "reduced_arrived_us": ag, "norm_done_us": norm,
               "max_us": [mx(3 + 4 * tt), mx(4 + 4 * tt), mx(5 + 4 * tt), mx(6 + 4 * tt)]}
        if k > 1 and arr is not None and norm is not None:
            if kind == "direct":
                row["nvlink_gbs"] = part_bytes / max(norm - arr, 1e-3) / 1e3
            elif stored is not None and ag is not None:
                row["rs_nvlink_gbs"] = slice_bytes / max(stored - arr, 1e-3) / 1e3
                row["ag_nvlink_gbs"] = slice_bytes / max(norm - ag, 1e-3) / 1e3
        out["tiles"].append(row)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--k", type=int, default=2)
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--relay", choices=["direct", "rsag"], default=None)
    ap.add_argument("--config", default="qwen2.5-7b")
    ap.add_argument("--seq", type=int, default=2048)
    ap.add_argument("--tiles", type=int, default=4)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--out")
    ap.add_argument("--raw", help="also save every CTA's raw trace slots (.npz, one array per rank)")
    args = ap.parse_args()
    traces, status, kind, stages, cfg = run(args.k, args.layers, args.relay, args.config, args.seq,
                                            args.tiles, args.iters)
    R = args.seq // args.tiles
    res = {"k": args.k, "relay": kind, "tiles": args.tiles, "seq": args.seq, "H": cfg.H,
           "status": status, "ranks": [], "stage_times": stages}
    for r, tr in enumerate(traces):
        s = summarise(tr, args.k, args.tiles, R, cfg.H, kind)
        res["ranks"].append(s)
        print(f"rank {r} ({kind}): GEMM epilogue done {s['gemm_done_us']:.1f} us, relay end "
              f"{s['relay_end_us']:.1f} us")
        for row in s["tiles"]:
            extra = ""
            if "nvlink_gbs" in row:
                extra = f"  pull {row['nvlink_gbs']:.0f} GB/s"
            elif "rs_nvlink_gbs" in row:
                extra = f"  RS {row['rs_nvlink_gbs']:.0f} GB/s, AG {row['ag_nvlink_gbs']:.0f} GB/s"
            fmt = lambda v: "   -  " if v is None else f"{v:6.1f}"
            print(f"  tile {row['tile']}: partials {fmt(row['partials_arrived_us'])}  stored "
                  f"{fmt(row['reduced_stored_us'])}  reduced {fmt(row['reduced_arrived_us'])}  norm "
                  f"{fmt(row['norm_done_us'])}{extra}  (latest CTA: "
                  + " ".join(fmt(v) for v in row["max_us"]) + ")")
        for sg in s["signals"]:
            print(f"  signal {sg['kind']} tile {sg['tile']}: local counter complete "
                  f"{sg['local_done_us']:6.1f}, forwarded {sg['forwarded_us']:6.1f} "
                  f"(fence + {args.k} adds {sg['fence_us']:.1f} us)")
    if args.out:
        Path(args.out).write_text(json.dumps(res, indent=1), encoding="utf-8")
    if args.raw:
        np.savez_compressed(args.raw, **{f"rank{r}": tr for r, tr in enumerate(traces)})
    if any(status):
        raise SystemExit(f"device status {status}")


if __name__ == "__main__":
    main()
