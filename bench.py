#!/usr/bin/env python3
"""Benchmark: Qwen2.5-7B-architecture prefill (S=2048) on N B200s, tp_split vs tp.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N=1 runs in-process; N>1 is launched by torchrun, one rank per GPU.  Each rank
creates a libkernrelay engine (C ABI, include/kernrelay_b200.h) for
  * tp{N}_split  -- the product: fused down-GEMM + NVLink relay + Add+RMSNorm
  * tp{N}        -- the unfused baseline: down GEMM -> NCCL AllReduce -> Add+RMSNorm
and times K CUDA-graph replays of the whole prefill per mode with CUDA events on
the engine stream, bracketed by a barrier and device synchronisation, taking
the max over ranks.  One step = one complete prefill of one 2048-token sequence
(every layer, lm_head over all 2048 rows on rank 0), so tokens/s = 2048 / step
time for the whole job (strong scaling: N GPUs share the same sequence).

Printed: one JSON line on rank 0 (value = tp_split tok/s).  `e2e` is the same
prefill through krb_engine_run_host (token ids copied from pinned host memory,
last-row logits copied back, inside the timed region).  `roofline`/`stages`
come from instrumented prefills (CUDA events between stages, same process,
after the timed region).  `cpu_baseline` (N=1, rank 0) times one complete fp32
prefill of the same workload with the CPU oracle port (oracle/cpu_sample.py).

--impl reference runs the reference arm: the CPU oracle port (the reference has
no runnable CPU or B200 implementation; its runtime needs Ascend/CANN), all host
threads, each step one complete prefill; under torchrun only rank 0 runs.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import timedelta
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))
# stdout carries exactly one JSON line: keep NCCL's banner off it
os.environ.setdefault("NCCL_DEBUG", "WARN")

METRIC = "Qwen2.5-7B prefill tok/s @seq2048 at 1/2/4/8 B200; tp_split vs tp speedup"
# the other BASELINE configurations (Qwen3-VL text decoders) report the same quantity
MODEL_NAMES = {
    "qwen2.5-7b": "Qwen2.5-7B architecture (28 layers, H 3584, I 18944, 28/4 heads, V 152064)",
    "qwen3-vl-4b": "Qwen3-VL-4B text decoder (36 layers, H 2560, I 9728, 32/8 heads, QK-norm, V 151936 tied)",
    "qwen3-vl-8b": "Qwen3-VL-8B text decoder (36 layers, H 4096, I 12288, 32/8 heads, QK-norm, V 151936)",
    "qwen2.5-0.5b": "Qwen2.5-0.5B architecture (24 layers, H 896, I 4864, 14/2 heads, V 151936 tied)",
}


def metric_for(config: str, S: int) -> str:
    if config == "qwen2.5-7b" and S == 2048:
        return METRIC
    return f"{config} prefill tok/s @seq{S} at 1/2/4/8 B200; tp_split vs tp speedup"
# the reference's published prefill times for this metric (Ascend 910B3, real weights): 146.2 ms
# single-device and 118.153 ms tp2 at S = 2048 -> tokens/s
PUBLISHED_TOKS = {1: 2048 / 0.1462, 2: 2048 / 0.118153}
NVLINK_SPEC_GBS = 900.0       # NVLink 5 per direction per GPU (nominal)
NVLINK_FALLBACK_GBS = 770.0   # earlier peer-copy measurement on this pool; used only at N = 1


def peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "tflops": d["bf16_tflops"],
                "tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "tflops": 1590.0, "tflops_sustained": 1400.0, "source": "fallback"}


# ------------------------------------------------------------------ distributed helpers
class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None
        self.backend = "nccl"
        self.nvlink = None   # peer-copy measurement (rank 0's, shared after init)

    def init(self, backend: str | None = None, timeout_s: float | None = None):
        """One process group per job: NCCL on GPUs (the driver's contract); gloo is
        accepted for the CPU tests of the host-side exchange logic.  A collective that a
        peer never joins fails after timeout_s (KRB_DIST_TIMEOUT_S, default 300 s)."""
        import torch
        import torch.distributed as dist
        self.backend = backend or os.environ.get("KRB_DIST_BACKEND", "nccl")
        if timeout_s is None:
            timeout_s = float(os.environ.get("KRB_DIST_TIMEOUT_S", "300"))
        if self.backend == "nccl":
            torch.cuda.set_device(self.local)
        if self.world > 1:
            kw = {"device_id": torch.device(f"cuda:{self.local}")} if self.backend == "nccl" else {}
            dist.init_process_group(self.backend, timeout=timedelta(seconds=timeout_s), **kw)
            self.pg = dist

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, v: float) -> float:
        if not self.pg:
            return v
        import torch
        dev = f"cuda:{self.local}" if self.backend == "nccl" else "cpu"
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def gather_bytes(self, b: bytes) -> list[bytes]:
        if not self.pg:
            return [b]
        out = [None] * self.world
        self.pg.all_gather_object(out, b)
        return out

    def bcast_bytes(self, b: bytes | None) -> bytes:
        if not self.pg:
            return b
        obj = [b]
        self.pg.broadcast_object_list(obj, src=0)
        return obj[0]

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


def pickle_bcast(d: Dist, obj):
    """rank 0's object on every rank (json over the byte broadcast)"""
    b = d.bcast_bytes(json.dumps(obj).encode() if d.rank == 0 else None)
    return json.loads(b.decode())


# ------------------------------------------------------------------ clocks
class Clocks:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.proc = None
        self.lines = []
        try:
            import torch
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            self.sel = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
        except Exception:
            self.sel = str(device)

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50", "-i", self.sel], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if not self.proc:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = [ln.split(",") for ln in out.strip().splitlines() if ln.count(",") >= 8]
        if not rows:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        pw = [float(r[3]) for r in rows if r[3].strip().replace(".", "").isdigit()]
        reasons = sorted({names[i] for r in rows for i in range(4) if "Active" in r[5 + i]
                          and "Not" not in r[5 + i]})
        loaded = [s for s, p in zip(sm, pw) if p > 300] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": max(mx) if mx else None, "power_w_max": max(pw) if pw else None,
                "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------------ workload model
def workload_name(config: str, S: int) -> str:
    """The workload both arms report in config.workload (same string, same work)."""
    return f"{config} prefill S={S} batch 1"


def model_dir(cfg_name: str, seq: int, seed: int, d: Dist, layers: int | None = None) -> Path:
    """Synthetic model directory (manifest + small tensors; large ones generated on the GPU)."""
    from kernrelay_b200 import model_gen
    root = Path(os.environ.get("KRB_MODEL_CACHE", tempfile.gettempdir())) / "krb_models"
    cfg = model_gen.CONFIGS[cfg_name]
    if layers:
        cfg = model_gen.config_with(cfg_name, L=layers)
    out = root / f"{cfg_name}_L{cfg.L}_s{seq}_seed{seed}_synth"
    if d.rank == 0 and not (out / "manifest.json").exists():
        tmp = root / f".{out.name}.{os.getpid()}"
        model_gen.write_model(tmp, cfg, seq, seed=seed, materialize=False)
        os.replace(tmp, out) if not out.exists() else None
    d.barrier()
    return out


def stage_work(cfg, S: int, k: int, rank: int):
    """Algorithmic work of each engine stage: (kind, amount per prefill, unit)."""
    H, D, HQ, HKV, V, L = cfg.H, cfg.D, cfg.HQ, cfg.HKV, cfg.V, cfg.L
    Iloc = cfg.I // k
    nqkv = (HQ + 2 * HKV) * D
    w = {
        "qkv": ("tensor", L * 2.0 * S * H * nqkv),
        "attention": ("tensor", L * 2.0 * S * S * D * HQ),   # causal half of 4*S^2*D*HQ
        "o": ("tensor", L * 2.0 * S * HQ * D * H),
        "gateup": ("tensor", L * 2.0 * S * H * 2 * Iloc),
        "rope": ("hbm", L * 2.0 * S * (HQ + HKV) * D * 2),
        "addnorm": ("hbm", L * (4 + 2 + 4 + 2) * S * H * 1.0),  # fp32 res in/out, bf16 delta, bf16 x
        "embed": ("hbm", S * H * (2 + 4 + 4 + 2) * 1.0),
    }
    if rank == 0:
        w["lm_head"] = ("tensor", 2.0 * S * H * V)
    return w


def relay_roofline_s(cfg, S, k, pk, nvlink_gbs):
    """Stage roofline of down+reduction: max(GEMM at tensor peak, bytes over NVLink)."""
    gemm = 2.0 * S * (cfg.I // k) * cfg.H / (pk["tflops_sustained"] * 1e12)
    comm = 2.0 * (k - 1) / k * S * cfg.H * 2 / (nvlink_gbs * 1e9)
    return max(gemm, comm), gemm, comm


def measure_peer_gbs(d: Dist, nbytes: int = 1 << 30, reps: int = 8):
    """Peer-copy bandwidth GPU 0 -> GPU 1 and back (copy engines over NVLink), per
    direction, measured by rank 0 before the process group exists (the other ranks are
    still in its rendezvous, with no kernel of theirs on a GPU).  Device events on the
    copying stream, after one warm-up copy; the best of two rounds per direction."""
    import torch
    gbs = None
    if d.rank == 0 and d.world > 1 and torch.cuda.device_count() >= 2:
        res = []
        for a, b in ((0, 1), (1, 0)):
            src = torch.empty(nbytes, dtype=torch.uint8, device=f"cuda:{a}")
            dst = torch.empty(nbytes, dtype=torch.uint8, device=f"cuda:{b}")
            with torch.cuda.device(b):
                s = torch.cuda.current_stream()
                dst.copy_(src)
                best = 0.0
                for _ in range(2):
                    torch.cuda.synchronize(a)
                    torch.cuda.synchronize(b)
                    e0, e1 = (torch.cuda.Event(enable_timing=True),
                              torch.cuda.Event(enable_timing=True))
                    e0.record(s)
                    for _ in range(reps):
                        dst.copy_(src, non_blocking=True)
                    e1.record(s)
                    e1.synchronize()
                    best = max(best, nbytes * reps / (e0.elapsed_time(e1) * 1e-3) / 1e9)
                res.append(best)
            torch.cuda.synchronize(a)
            del src, dst
        torch.cuda.empty_cache()
        gbs = {"gpu0_to_gpu1_gbs": round(res[0], 1), "gpu1_to_gpu0_gbs": round(res[1], 1),
               "per_direction_gbs": round(min(res), 1), "spec_gbs": NVLINK_SPEC_GBS,
               "how": f"torch peer copy of {nbytes >> 20} MiB x {reps}, CUDA events, best of 2"}
    return gbs


# ------------------------------------------------------------------ our arm
def run_mode(d: Dist, mdir: Path, mode: str, S: int, tiles: int, K: int, W: int, e2e: bool,
             clocks: Clocks | None):
    import numpy as np
    import torch
    from kernrelay_b200._lib import Engine
    eng = Engine(mdir, mode, S, rank=d.rank, world=d.world, device=d.local, tiles=tiles)
    try:
        if "split" in mode and d.world > 1:
            eng.open_peers(d.gather_bytes(eng.ipc_handle()))
        elif d.world > 1:
            uid = d.bcast_bytes(Engine.nccl_unique_id() if d.rank == 0 else None)
            eng.init_nccl(uid)
        d.barrier()
        eng.run()           # first (direct) run: loads caches, checks status
        eng.sync()
        eng.capture()       # whole prefill as one CUDA graph
        stream = torch.cuda.ExternalStream(eng.stream_ptr(), device=d.local)
        for _ in range(W):
            eng.run()
        eng.sync()
        torch.cuda.synchronize()
        d.barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        if clocks:
            clocks.start()
        torch.cuda.synchronize()
        d.barrier()
        torch.cuda.nvtx.range_push("krb_timed")  # lets a profiler select the timed replays
        e0.record(stream)
        for _ in range(K):
            eng.run()
        e1.record(stream)
        torch.cuda.nvtx.range_pop()
        eng.sync()
        torch.cuda.synchronize()
        d.barrier()
        ck = clocks.stop() if clocks else None
        ms = d.max(e0.elapsed_time(e1)) / K
        res = {"mode": mode, "ms_per_step": ms, "clocks": ck}
        st = eng.status()
        if st:
            raise RuntimeError(f"{mode}: device status {st}")
        info = eng.info()
        res["launches_per_run"] = info["launches_per_run"]
        res["relay"] = info.get("relay")
        if d.rank == 0:
            logits = eng.last_logits()
            res["argmax"] = int(np.argmax(logits))
            res["finite"] = bool(np.isfinite(logits).all())
        if e2e:
            V = info["V"]
            ids = torch.from_numpy(np.fromfile(mdir / "ids.bin", dtype=np.int64)).pin_memory()
            logits_h = torch.empty(V, dtype=torch.float32).pin_memory() if d.rank == 0 else None
            for _ in range(max(1, W)):
                eng.run_host(ids, logits_h)
            eng.sync()
            d.barrier()
            torch.cuda.synchronize()
            e0.record(stream)
            for _ in range(K):
                eng.run_host(ids, logits_h)
            e1.record(stream)
            eng.sync()
            d.barrier()
            ems = d.max(e0.elapsed_time(e1)) / K
            res["e2e"] = {"ms_per_step": ems, "h2d_bytes_per_step": int(ids.numel() * 8),
                          "d2h_bytes_per_step": int(V * 4) if d.rank == 0 else 0}
            if d.rank == 0:
                res["e2e_argmax"] = int(np.argmax(logits_h.numpy()))
        # per-stage device times from instrumented (event-bracketed) prefills
        stages = None
        for _ in range(3):
            t = eng.stage_times()["stage_us"]
            stages = t if stages is None else {k: stages[k] + t[k] for k in t}
        res["stage_us"] = {k: v / 3 for k, v in stages.items()}
        d.barrier()
        return res
    finally:
        eng.close()


def roofline_block(cfg, S, k, rank, split_res, pk, nvlink_gbs=NVLINK_FALLBACK_GBS,
                   config_name="qwen2.5-7b"):
    st = split_res["stage_us"]
    work = stage_work(cfg, S, k, rank)
    stages = {}
    for name, (kind, amount) in work.items():
        us = st.get(name, 0.0)
        if us <= 0:
            continue
        if kind == "tensor":
            ach = amount / (us * 1e-6) / 1e12
            peak = pk["tflops_sustained"]
            stages[name] = {"us": round(us, 1), "achieved": round(ach, 1), "peak": peak,
                            "unit": "TFLOP/s", "frac": round(ach / peak, 3)}
        else:
            ach = amount / (us * 1e-6) / 1e9
            stages[name] = {"us": round(us, 1), "achieved": round(ach, 1), "peak": pk["hbm_gbs"],
                            "unit": "GB/s", "frac": round(ach / pk["hbm_gbs"], 3)}
    if "o" in stages and st.get("addnorm", 0.0) <= 0:
        # the tp modes run o_proj, the residual add and ln2 as one kernel: its time (and
        # the fraction, against the GEMM's flops alone) includes the Add+RMSNorm
        stages["o"]["includes"] = "residual add + ln2 RMSNorm (one kernel)"
    relay_us = st.get("relay", 0.0)
    if relay_us > 0:
        roof_s, gemm_s, comm_s = relay_roofline_s(cfg, S, k, pk, nvlink_gbs)
        flops = cfg.L * 2.0 * S * (cfg.I // k) * cfg.H
        stages["relay"] = {"us": round(relay_us, 1), "roofline_us": round(cfg.L * roof_s * 1e6, 1),
                           "frac": round(cfg.L * roof_s * 1e6 / relay_us, 3),
                           "achieved": round(flops / (relay_us * 1e-6) / 1e12, 1),
                           "unit": "TFLOP/s", "bound": "tensor" if gemm_s >= comm_s else "nvlink",
                           "nvlink_gbs": nvlink_gbs}
    # dominant kernel by time share
    dom = max(stages.items(), key=lambda kv: kv[1]["us"])
    name, s = dom
    if name == "relay":
        flops_per_launch = 2.0 * S * (cfg.I // k) * cfg.H
        launch_us = s["us"] / cfg.L
        roof = {"kernel": "relay_down_kernel (down GEMM + relay + Add+RMSNorm)", "bound": "tensor",
                "achieved": round(flops_per_launch / (launch_us * 1e-6) / 1e12, 1),
                "peak": pk["tflops_sustained"], "unit": "TFLOP/s"}
    else:
        kind, amount = work[name]
        launches = 1 if name in ("lm_head", "embed") else cfg.L
        launch_us = s["us"] / launches
        per = amount / launches
        if kind == "tensor":
            roof = {"kernel": name, "bound": "tensor", "achieved": round(per / (launch_us * 1e-6) / 1e12, 1),
                    "peak": pk["tflops_sustained"], "unit": "TFLOP/s"}
        else:
            roof = {"kernel": name, "bound": "hbm", "achieved": round(per / (launch_us * 1e-6) / 1e9, 1),
                    "peak": pk["hbm_gbs"], "unit": "GB/s"}
    roof["frac"] = round(roof["achieved"] / roof["peak"], 3)
    roof["traffic"] = traffic_for(config_name, S, name, k)
    roof["peak_source"] = f"{pk['source']} ({'sustained bf16' if roof['unit'] == 'TFLOP/s' else 'HBM copy'})"
    roof["launch_us"] = round(launch_us, 2)
    return roof, stages


def traffic_for(config: str, S: int, stage: str, k: int):
    """DRAM bytes (read + write) per launch of `stage` at tp degree k for model `config` at
    sequence length S, from the committed ncu summary (profiles/traffic.txt, lines
    `config/S/stage@k = bytes`), or None if that case was not captured."""
    p = REPO / "profiles" / "traffic.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("#") or not line.strip():
            continue
        name, _, val = line.partition("=")
        if name.strip() == f"{config}/{S}/{stage}@{k}":
            try:
                return float(val.split()[0])
            except ValueError:
                return None
    return None


def cpu_baseline(cfg, S, k):
    """One complete fp32 prefill of the same workload on the host cores (rank 0, N=1):
    about 15-20 s on a 16-core host.  A one-layer call warms the allocator first."""
    from oracle.cpu_sample import CpuPrefill, cpu_info
    cp = CpuPrefill(cfg, S, tp=k, threads=os.cpu_count())
    h = cp.w["lm"].t()[cp.ids]
    cp.layer(h, h)
    secs, top = cp.step()
    out = {"value": round(S / secs, 2), "unit": "tok/s", "cores": cp.threads, "kind": "port",
           "sample": cp.describe() + "; 1 timed prefill", "prefill_s": round(secs, 3)}
    out.update(cpu_info())
    return out


def run_ours(args, d: Dist):
    import torch
    from kernrelay_b200 import build, model_gen
    if not os.environ.get("KRB_NO_BUILD"):
        if d.rank == 0:
            build.build()
        d.barrier()
    cfg = model_gen.CONFIGS[args.config]
    if args.layers:
        cfg = model_gen.config_with(args.config, L=args.layers)
    S, N = args.seq, d.world
    mdir = model_dir(args.config, S, args.seed, d, args.layers)
    pk = peaks()
    nvlink = d.nvlink if N > 1 else None
    nvlink_gbs = nvlink["per_direction_gbs"] if nvlink else NVLINK_FALLBACK_GBS
    clocks = Clocks(d.local) if d.rank == 0 else None
    split = run_mode(d, mdir, f"tp{N}_split", S, args.tiles, args.steps, args.warmup, True, clocks)
    base = None
    if not args.no_tp:
        base = run_mode(d, mdir, f"tp{N}", S, 1, args.steps, args.warmup, False, None)
    pp = run_pp2(d, mdir, S, args) if args.pp2 else None
    if d.rank != 0:
        return None
    toks = S / (split["ms_per_step"] * 1e-3)
    roof, stages = roofline_block(cfg, S, N, 0, split, pk, nvlink_gbs, args.config)
    line = {
        "metric": metric_for(args.config, S),
        "value": round(toks, 1),
        "unit": "tok/s",
        "n_gpus": N,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(split["ms_per_step"], 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": (round(toks / PUBLISHED_TOKS[N], 3)
                        if N in PUBLISHED_TOKS and metric_for(args.config, S) == METRIC else None),
        "dtype": "fp16",
        "precision": ("weights bf16 (the model's dtype) converted exactly to fp16 at load; GEMM and "
                      "attention operands and activations fp16 (8x finer rounding than bf16, same "
                      "tensor-core rate); fp32 accumulation, fp32 residual stream"),
        "data": "synthetic: seeded random-init weights N(0,0.02) (norms 1), uniform random token ids (seed 1234)",
        "config": {"workload": workload_name(args.config, S)
                               + (f" (PROFILING: {cfg.L} layers)" if args.layers else ""),
                   "model": MODEL_NAMES.get(args.config, args.config),
                   "global_batch": 1, "seq_len": S, "parallelism": f"tp{N} MLP (attention replicated)",
                   "mode": split["mode"], "tiles": args.tiles, "graph": True,
                   "relay_form": split.get("relay"),
                   "lm_head_rows": S,
                   "l2": "no flush needed: every step streams all weights (>=15 GB at tp1, >=4.5 GB per GPU at tp8) through the 126 MB L2"},
        "tp_baseline": None if base is None else {
            "mode": base["mode"], "ms_per_step": round(base["ms_per_step"], 4),
            "value": round(S / (base["ms_per_step"] * 1e-3), 1), "unit": "tok/s",
            "stage_us": {k_: round(v, 1) for k_, v in base["stage_us"].items()}},
        "speedup_tp_split_vs_tp": None if base is None else round(base["ms_per_step"] / split["ms_per_step"], 4),
        "e2e": {"value": round(S / (split["e2e"]["ms_per_step"] * 1e-3), 1), "unit": "tok/s",
                "ms_per_step": round(split["e2e"]["ms_per_step"], 4),
                "h2d_bytes_per_step": split["e2e"]["h2d_bytes_per_step"],
                "d2h_bytes_per_step": split["e2e"]["d2h_bytes_per_step"],
                "api": "krb_engine_run_host (ids H2D from pinned host, prefill, last-row logits D2H)"},
        "roofline": roof,
        "stages": stages,
        "nvlink": nvlink,
        "clocks": split.get("clocks"),
        "gpu_launches": int(split["launches_per_run"]) * args.steps,
        "argmax": split.get("argmax"),
        "argmax_tp_baseline": None if base is None else base.get("argmax"),
    }
    if N == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline(cfg, S, 1)
    if pp is not None:
        line["pp2_baseline"] = pp
    return line


def run_pp2(d: Dist, mdir: Path, S: int, args):
    """The PP=2 layer-pipeline baseline (reference RunQwenPP, qwen_main.cpp:1993-2146) on GPUs
    0 and 1 through kr_qwen_pp_run, one request (the reference's R=1 row), run by rank 0 after
    the TP measurement while the other ranks wait.  Host-timed wall per prefill, as the
    reference reports it."""
    import torch
    res = None
    if d.rank == 0:
        if torch.cuda.device_count() < 2:
            res = {"unavailable": "needs 2 visible GPUs"}
        else:
            from kernrelay_b200 import libapi
            r = libapi.qwen_pp_run(mdir, mode="pp", seq=S, dev0=0, dev1=1, requests=1,
                                   warmup=max(1, args.warmup), iters=max(3, args.steps // 4))
            if r.get("_rc") != 0:
                res = {"error": r.get("error", "kr_qwen_pp_run failed")}
            else:
                best = r["wall_best_us"]
                res = {"mode": r.get("mode"), "devices": r.get("devices"), "requests": 1,
                       "layers": r.get("layers"), "wall_best_us": best,
                       "wall_typical_us": r.get("wall_typical_us"),
                       "value": round(S / (best * 1e-6), 1), "unit": "tok/s",
                       "timing": "host wall per prefill (enqueue + device), best of iters"}
    d.barrier()
    return res


# ------------------------------------------------------------------ micro-DAG workload
MICRODAG_METRIC = ("TP-MLP micro-DAG step time (down GEMM -> AllReduce -> Add+RMSNorm, 4 row tiles) "
                   "at 1/2/4/8 B200; tp_split vs tp")


def _microdag_engine(d: Dist, mode: str, S: int, H: int, I: int, tiles: int, seed: int):
    from kernrelay_b200._lib import Engine
    eng = Engine.microdag(S, H, I, mode, rank=d.rank, world=d.world, device=d.local, tiles=tiles,
                          seed=seed)
    if d.world > 1:
        if "split" in mode:
            eng.open_peers(d.gather_bytes(eng.ipc_handle()))
        else:
            uid = d.bcast_bytes(Engine.nccl_unique_id() if d.rank == 0 else None)
            eng.init_nccl(uid)
    d.barrier()
    return eng


def time_microdag(d: Dist, eng, K: int, W: int, clocks: Clocks | None):
    """K steps of [L2 flush (a 512 MiB device write; at k >= 4 a rank's operands fit in the
    126 MB L2), one micro-DAG step (graph replay)] back to back on the engine stream, timed
    by CUDA events around the whole loop, minus K flushes alone timed the same way right
    after (W warm-up steps in the same pattern first touch the flush buffer).  The
    ranks stay in step without a host barrier per step (every relay step waits for its
    peers), so a per-step flush does not shift the ranks against each other.  Returns the
    per-step time, max over ranks (ms)."""
    import torch
    eng.run()
    eng.sync()
    eng.capture()
    stream = torch.cuda.ExternalStream(eng.stream_ptr(), device=d.local)
    flush = torch.empty(512 << 20, dtype=torch.uint8, device=f"cuda:{d.local}")
    e = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    with torch.cuda.stream(stream):
        # warm-up: the flush buffer's first writes and W steps in the timed pattern
        for i in range(W):
            flush.fill_(i & 0xFF)
            eng.run()
        eng.sync()
        torch.cuda.synchronize()
        d.barrier()
        if clocks:
            clocks.start()
        torch.cuda.synchronize()
        d.barrier()
        e[2].record(stream)
        for i in range(K):
            flush.fill_(i & 0xFF)
            eng.run()
        e[3].record(stream)
        eng.sync()
        torch.cuda.synchronize()
        d.barrier()
        # the same K flushes alone, right after (same clocks and memory state)
        e[0].record(stream)
        for i in range(K):
            flush.fill_(i & 0xFF)
        e[1].record(stream)
    eng.sync()
    torch.cuda.synchronize()
    d.barrier()
    ck = clocks.stop() if clocks else None
    flush_ms = e[0].elapsed_time(e[1]) / K
    step_ms = d.max(e[2].elapsed_time(e[3]) / K - flush_ms)
    if step_ms <= 0:
        raise RuntimeError(f"micro-DAG: step time {step_ms:.4f} ms after subtracting the flush "
                           f"({flush_ms:.4f} ms): timing is not usable")
    st = eng.status()
    if st:
        raise RuntimeError(f"micro-DAG: device status {st}")
    stages = None
    for _ in range(3):
        t = eng.stage_times()["stage_us"]
        stages = t if stages is None else {k: stages[k] + t[k] for k in t}
    return step_ms, ck, {k: v / 3 for k, v in stages.items()}, flush_ms


def run_microdag(args, d: Dist):
    """X [S, I/k], W [I/k, H] per rank, R [S, H], gamma 1, T row tiles."""
    from kernrelay_b200 import build, model_gen
    if not os.environ.get("KRB_NO_BUILD"):
        if d.rank == 0:
            build.build()
        d.barrier()
    cfg = model_gen.CONFIGS[args.config]
    S, H, I, N = args.seq, cfg.H, cfg.I, d.world
    pk = peaks()
    nvlink = d.nvlink if N > 1 else None
    nvlink_gbs = nvlink["per_direction_gbs"] if nvlink else NVLINK_FALLBACK_GBS
    clocks = Clocks(d.local) if d.rank == 0 else None
    res = {}
    for mode in (f"tp{N}_split", f"tp{N}"):
        if mode == f"tp{N}" and args.no_tp:
            continue
        eng = _microdag_engine(d, mode, S, H, I, args.tiles, args.seed)
        try:
            ms, ck, st, fl = time_microdag(d, eng, args.steps, args.warmup,
                                           clocks if "split" in mode else None)
            res[mode] = {"ms": ms, "clocks": ck, "stage_us": st, "flush_ms": fl,
                         "launches": eng.info()["launches_per_run"]}
        finally:
            eng.close()
        d.barrier()
    if d.rank != 0:
        return None
    split = res[f"tp{N}_split"]
    cfg1 = model_gen.config_with(args.config, L=1)
    roof_s, gemm_s, comm_s = relay_roofline_s(cfg1, S, N, pk, nvlink_gbs)
    us = split["ms"] * 1e3
    flops = 2.0 * S * (I // N) * H
    line = {
        "metric": MICRODAG_METRIC, "value": round(us, 2), "unit": "us", "n_gpus": N,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(split["ms"], 5),
        "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "fp16",
        "precision": "X, W bf16 values held in fp16; fp32 accumulation; partials fp16 (k > 1)",
        "data": "synthetic: X ~ N(0,1), W ~ N(0,0.02) (seed 1234 + rank), R ~ N(0,1), gamma 1",
        "config": {"workload": f"microdag S={S} H={H} I={I}/k T={args.tiles}",
                   "model": "isolated TP-MLP micro-DAG (BASELINE configs[1])", "seq_len": S,
                   "global_batch": 1, "parallelism": f"tp{N}", "graph": True,
                   "l2": ("flushed before every step: a 512 MiB write; the same loop of writes "
                          "alone is timed and subtracted (flush_us)"),
                   "flush_us": round(split["flush_ms"] * 1e3, 2)},
        "roofline": {"stage": "down GEMM + reduction + Add+RMSNorm", "roofline_us": round(roof_s * 1e6, 2),
                     "gemm_us_at_peak": round(gemm_s * 1e6, 2), "nvlink_us": round(comm_s * 1e6, 2),
                     "bound": "tensor" if gemm_s >= comm_s else "nvlink",
                     "frac": round(roof_s * 1e6 / us, 3),
                     "achieved": round(flops / (us * 1e-6) / 1e12, 1), "unit": "TFLOP/s",
                     "peak": pk["tflops_sustained"],
                     "peak_source": f"{pk['source']} (sustained bf16)", "nvlink_gbs": nvlink_gbs},
        "nvlink": nvlink,
        "clocks": split["clocks"],
        "gpu_launches": split["launches"] * args.steps,
        "stage_us": {k: round(v, 1) for k, v in split["stage_us"].items() if v},
    }
    if f"tp{N}" in res:
        base = res[f"tp{N}"]
        line["tp_baseline"] = {"mode": f"tp{N}", "us": round(base["ms"] * 1e3, 2),
                               "frac": round(roof_s / (base["ms"] * 1e-3), 3),
                               "stage_us": {k: round(v, 1) for k, v in base["stage_us"].items() if v}}
        line["speedup_tp_split_vs_tp"] = round(base["ms"] / split["ms"], 4)
    return line


# ------------------------------------------------------------------ reference arm
def run_reference(args):
    """The reference arm: the fp32 CPU port of the reference prefill, timed on the host
    cores with every thread, each step one complete prefill of the workload (no sampling,
    no extrapolation).  If K + W prefills would not fit KRB_REF_BUDGET_S (default 900 s),
    fewer timed steps run and the line reports the count that ran."""
    from kernrelay_b200 import model_gen
    from oracle.cpu_sample import CpuPrefill, cpu_info
    cfg = model_gen.CONFIGS[args.config]
    S, N = args.seq, args.gpus
    budget = float(os.environ.get("KRB_REF_BUDGET_S", "900"))
    t_start = time.perf_counter()
    cp = CpuPrefill(cfg, S, tp=1, threads=os.cpu_count())
    warm = []
    for _ in range(max(0, args.warmup)):
        warm.append(cp.step()[0])
    per = min(warm) if warm else None
    steps = args.steps
    if per is not None:
        left = budget - (time.perf_counter() - t_start)
        steps = max(1, min(args.steps, int(left // per)))
    times = []
    top = None
    for _ in range(steps):
        secs, top = cp.step()
        times.append(secs)
    wall = sum(times)
    ms = wall / len(times) * 1e3
    toks = S / (ms * 1e-3)
    cb = {"value": round(toks, 2), "unit": "tok/s", "cores": cp.threads, "kind": "port",
          "sample": cp.describe() + f"; {len(times)} timed prefills, mean"}
    cb.update(cpu_info())
    line = {
        "metric": metric_for(args.config, S), "impl": "reference", "value": round(toks, 2),
        "unit": "tok/s",
        "n_gpus": N, "steps": len(times), "warmup": len(warm),
        "ms_per_step": round(ms, 2), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "fp32", "data": "synthetic (random weights of the exact shapes)",
        "config": {"workload": workload_name(args.config, S),
                   "model": MODEL_NAMES.get(args.config, args.config),
                   "seq_len": S, "global_batch": 1, "parallelism": "none (host CPU)"},
        "cpu_baseline": cb,
        "e2e": {"value": round(toks, 2), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": ("the reference runtime targets Ascend 910B3/CANN and cannot run here; the reference arm "
                 "is the fp32 CPU restatement of its prefill, each step a complete prefill"),
        "timed_wall_s": round(wall, 2),
        "last_row_argmax": top,
    }
    if len(times) != args.steps:
        line["steps_requested"] = args.steps
    return line


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", default="qwen2.5-7b")
    ap.add_argument("--seq", type=int, default=2048)
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--tiles", type=int, default=4)
    ap.add_argument("--no-tp", action="store_true", help="skip the NCCL tp baseline")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--layers", type=int, default=None,
                    help="profiling only: fewer decoder layers (not a valid benchmark number)")
    ap.add_argument("--pp2", action="store_true",
                    help="also time the PP=2 layer-pipeline baseline on GPUs 0 and 1 (rank 0)")
    ap.add_argument("--workload", choices=["prefill", "microdag"], default="prefill",
                    help="prefill: the headline metric; microdag: BASELINE configs[1] (the "
                         "isolated down GEMM -> AllReduce -> AddNorm stage)")
    args = ap.parse_args()
    d = Dist()
    if args.impl == "reference":
        if d.rank != 0:
            return 0
        print(json.dumps(run_reference(args)), flush=True)
        return 0
    if d.world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={d.world}")
    d.nvlink = measure_peer_gbs(d)   # rank 0, before any collective exists
    d.init()
    if d.world > 1:
        d.nvlink = pickle_bcast(d, d.nvlink)
    try:
        line = run_microdag(args, d) if args.workload == "microdag" else run_ours(args, d)
        if line is not None:
            print(json.dumps(line), flush=True)
    finally:
        d.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
