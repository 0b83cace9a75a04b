"""Timed CPU baseline for bench.py -- TEST INFRASTRUCTURE ONLY (the "port" arm).

The reference has no CPU prefill of its own; its oracle is HF transformers
(scripts/export_model.py:211-223), which oracle/qwen_ref.py restates in torch
fp32.  A full 7B prefill at S=2048 is ~30 TFLOP, minutes on a host CPU, so the
timed baseline runs a bounded SAMPLE of the same workload with the oracle's own
op functions and extrapolates:

    one decoder layer at full S (QKV+bias, RoPE, causal GQA attention, O,
    Add+RMSNorm, SiLU-gated MLP sharded like rank 0 of tp k, Add+RMSNorm)
    + the lm_head on V/vocab_div vocabulary columns over all S rows
    prefill_time ~= L * t_layer + vocab_div * t_lm_slice

Weights are random tensors of the exact shapes (timing does not depend on
their values).  Returned tok/s = S / prefill_time.
"""
from __future__ import annotations

import math
import os
import time

from .qwen_ref import apply_rope, causal_gqa, rmsnorm


def _shapes(cfg):
    return dict(H=cfg.H, I=cfg.I, L=cfg.L, HQ=cfg.HQ, HKV=cfg.HKV, D=cfg.D, V=cfg.V)


class CpuSample:
    def __init__(self, cfg, seq: int, tp: int = 1, threads: int | None = None, vocab_div: int = 16,
                 seed: int = 0):
        import torch
        self.torch = torch
        if threads:
            torch.set_num_threads(threads)
        self.threads = torch.get_num_threads()
        g = torch.Generator().manual_seed(seed)
        s = _shapes(cfg)
        self.cfg, self.S, self.tp, self.vocab_div = cfg, seq, tp, vocab_div
        H, D, HQ, HKV = s["H"], s["D"], s["HQ"], s["HKV"]
        Iloc = s["I"] // tp
        r = lambda *shape: torch.randn(*shape, generator=g) * 0.02  # noqa: E731
        self.w = dict(q=r(H, HQ * D), k=r(H, HKV * D), v=r(H, HKV * D), bq=r(HQ * D), bk=r(HKV * D),
                      bv=r(HKV * D), o=r(HQ * D, H), g=r(H, Iloc), u=r(H, Iloc), d=r(Iloc, H),
                      ln=torch.ones(H), lm=r(H, max(1, s["V"] // vocab_div)))
        ang = torch.outer(torch.arange(seq, dtype=torch.float64),
                          1.0 / (cfg.theta ** (torch.arange(0, D, 2, dtype=torch.float64) / D)))
        self.cos = torch.cat([ang.cos(), ang.cos()], -1).float()
        self.sin = torch.cat([ang.sin(), ang.sin()], -1).float()
        self.h = torch.randn(seq, H, generator=g)
        self.x = rmsnorm(self.h, self.w["ln"], cfg.eps)

    def layer(self):
        w, S, c = self.w, self.S, self.cfg
        x, h = self.x, self.h
        q = (x @ w["q"] + w["bq"]).view(S, c.HQ, c.D)
        k = (x @ w["k"] + w["bk"]).view(S, c.HKV, c.D)
        v = (x @ w["v"] + w["bv"]).view(S, c.HKV, c.D)
        q = apply_rope(q, self.cos, self.sin)
        k = apply_rope(k, self.cos, self.sin)
        a = causal_gqa(q, k, v, 1.0 / math.sqrt(c.D))
        h1 = h + a @ w["o"]
        x2 = rmsnorm(h1, w["ln"], c.eps)
        act = self.torch.nn.functional.silu(x2 @ w["g"]) * (x2 @ w["u"])
        h2 = h1 + act @ w["d"]
        return rmsnorm(h2, w["ln"], c.eps)

    def lm_slice(self):
        return self.x @ self.w["lm"]

    def step(self):
        """One bounded sample; returns (estimated prefill seconds, sample seconds)."""
        t0 = time.perf_counter()
        self.layer()
        t1 = time.perf_counter()
        self.lm_slice()
        t2 = time.perf_counter()
        est = self.cfg.L * (t1 - t0) + self.vocab_div * (t2 - t1)
        return est, t2 - t0

    def describe(self):
        return (f"1 of {self.cfg.L} decoder layers (tp{self.tp} rank-0 MLP shard) at S={self.S} "
                f"+ lm_head on 1/{self.vocab_div} of V={self.cfg.V}; prefill time = "
                f"L*t_layer + {self.vocab_div}*t_lm_slice; torch fp32, {self.threads} threads")


def cpu_info():
    model = ""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return {"cpu_model": model, "os_cpu_count": os.cpu_count()}
