"""Timed CPU prefill for bench.py -- TEST INFRASTRUCTURE ONLY (the "port" arm).

The reference has no CPU prefill of its own; its oracle is HF transformers
(scripts/export_model.py:211-223), which oracle/qwen_ref.py restates in torch
fp32.  This module times that restatement's op sequence over a COMPLETE prefill
of the benchmark configuration -- nothing is sampled or extrapolated:

    embed gather -> ln1_0 -> L x { QKV (+bias) [-> QK-norm] -> RoPE -> causal GQA
    attention -> O -> Add+RMSNorm -> SiLU-gated MLP (rank 0's shard of tp k) ->
    Add+RMSNorm } -> lm_head over all S rows (as the reference computes it,
    qwen_main.cpp:1305-1307)

One layer's random weights of the exact shapes are reused by all L layers (the
time of an fp32 matmul does not depend on the values), so the host holds one
layer plus the embedding / lm_head instead of the whole model.  The embedding
gather reads rows of the lm_head's transpose (the tied layout), which costs the
same S x H gather as a separate table.  Returned tok/s = S / prefill seconds.
"""
from __future__ import annotations

import math
import os
import time

from .qwen_ref import apply_rope, causal_gqa, rmsnorm


class CpuPrefill:
    def __init__(self, cfg, seq: int, tp: int = 1, threads: int | None = None, seed: int = 0):
        import torch
        self.torch = torch
        if threads:
            torch.set_num_threads(threads)
        self.threads = torch.get_num_threads()
        g = torch.Generator().manual_seed(seed)
        self.cfg, self.S, self.tp = cfg, seq, tp
        H, D, HQ, HKV = cfg.H, cfg.D, cfg.HQ, cfg.HKV
        Iloc = cfg.I // tp
        r = lambda *shape: torch.randn(*shape, generator=g) * 0.02  # noqa: E731
        self.w = dict(q=r(H, HQ * D), k=r(H, HKV * D), v=r(H, HKV * D), o=r(HQ * D, H),
                      g=r(H, Iloc), u=r(H, Iloc), d=r(Iloc, H), ln=torch.ones(H),
                      lm=r(H, cfg.V))
        if cfg.bias:
            self.w.update(bq=r(HQ * D), bk=r(HKV * D), bv=r(HKV * D))
        if cfg.qk_norm:
            self.w.update(qn=torch.ones(D), kn=torch.ones(D))
        ang = torch.outer(torch.arange(seq, dtype=torch.float64),
                          1.0 / (cfg.theta ** (torch.arange(0, D, 2, dtype=torch.float64) / D)))
        self.cos = torch.cat([ang.cos(), ang.cos()], -1).float()
        self.sin = torch.cat([ang.sin(), ang.sin()], -1).float()
        self.ids = torch.randint(0, cfg.V, (seq,), generator=g)

    def layer(self, h, x):
        w, S, c = self.w, self.S, self.cfg
        q, k, v = x @ w["q"], x @ w["k"], x @ w["v"]
        if c.bias:
            q, k, v = q + w["bq"], k + w["bk"], v + w["bv"]
        q, k, v = q.view(S, c.HQ, c.D), k.view(S, c.HKV, c.D), v.view(S, c.HKV, c.D)
        if c.qk_norm:
            q = rmsnorm(q, w["qn"], c.eps)
            k = rmsnorm(k, w["kn"], c.eps)
        q = apply_rope(q, self.cos, self.sin)
        k = apply_rope(k, self.cos, self.sin)
        a = causal_gqa(q, k, v, 1.0 / math.sqrt(c.D))
        h1 = h + a @ w["o"]
        x2 = rmsnorm(h1, w["ln"], c.eps)
        act = self.torch.nn.functional.silu(x2 @ w["g"]) * (x2 @ w["u"])
        h2 = h1 + act @ w["d"]
        return h2, rmsnorm(h2, w["ln"], c.eps)

    def step(self):
        """One complete prefill; returns (seconds, last-row argmax)."""
        t0 = time.perf_counter()
        h = self.w["lm"].t()[self.ids]
        x = rmsnorm(h, self.w["ln"], self.cfg.eps)
        for _ in range(self.cfg.L):
            h, x = self.layer(h, x)
        logits = x @ self.w["lm"]
        top = int(logits[-1].argmax())
        return time.perf_counter() - t0, top

    def describe(self):
        return (f"complete {self.cfg.L}-layer prefill at S={self.S} (tp{self.tp} rank-0 MLP shard), "
                f"lm_head over all {self.S} rows, V={self.cfg.V}; torch fp32, {self.threads} threads; "
                "one layer's random weights reused by every layer")


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
