"""Seeded random-init model directories in the reference's on-disk format.

The reference exports real Hugging Face checkpoints into
  manifest.json + weights.bin (bf16, matmul weights transposed to [K, N]) + ids.bin
  (+ ref_last_logits.bin / ref.json from the HF forward)
(scripts/export_model.py:142-223).  No checkpoint exists on a B200 box, so this
module writes the same layout for the random-init configurations of the
benchmark.  Weights are drawn from a counter-based generator (SplitMix64 ->
Irwin-Hall(12) ~ N(mean, std^2), rounded to bf16) that the CUDA loader can
evaluate on the device; `materialize=False` writes only the small tensors to
weights.bin and marks the large ones {"synth": {...}} in the manifest, so a 7B
model directory is a few MB and loads in seconds.

Token ids follow export_model.py:206-210 exactly: torch.randint(0, V, (1, S))
with torch.Generator().manual_seed(seed), stored int64.  RoPE tables follow
export_model.py:70-77 (float64 angles, cos/sin rounded to bf16, [1,1,max_pos,D]).
"""
from __future__ import annotations

import argparse
import json
from dataclasses import asdict, dataclass, replace
from pathlib import Path

import numpy as np


@dataclass(frozen=True)
class ModelConfig:
    arch: str
    H: int
    I: int
    L: int
    HQ: int
    HKV: int
    D: int
    V: int
    tied: bool
    bias: bool
    qk_norm: bool
    theta: float
    eps: float = 1e-6


CONFIGS = {
    # Qwen2.5-0.5B architecture
    "qwen2.5-0.5b": ModelConfig("qwen2.5", 896, 4864, 24, 14, 2, 64, 151936, True, True, False, 1e6),
    # Qwen2.5-7B architecture
    "qwen2.5-7b": ModelConfig("qwen2.5", 3584, 18944, 28, 28, 4, 128, 152064, False, True, False, 1e6),
    # Qwen3-VL-4B text decoder
    "qwen3-vl-4b": ModelConfig("qwen3_vl", 2560, 9728, 36, 32, 8, 128, 151936, True, False, True, 5e6),
    # Qwen3-VL-8B text decoder
    "qwen3-vl-8b": ModelConfig("qwen3_vl", 4096, 12288, 36, 32, 8, 128, 151936, False, False, True, 5e6),
    # test-sized shapes of both families
    "tiny-qwen2": ModelConfig("qwen2.5", 256, 512, 2, 4, 2, 64, 1024, True, True, False, 1e6),
    "tiny-qwen3": ModelConfig("qwen3_vl", 256, 768, 2, 2, 1, 128, 1024, False, False, True, 5e6),
    # the 0.5B head layout (14 / 2 heads of 64, GQA 7, QKV bias) at two layers
    "small-qwen2-gqa7": ModelConfig("qwen2.5", 896, 1024, 2, 14, 2, 64, 2048, True, True, False, 1e6),
    # Qwen3-VL head layout (GQA 4, head_dim 128, QK-norm, theta 5e6; q width != hidden)
    "small-qwen3-gqa4": ModelConfig("qwen3_vl", 512, 1024, 2, 8, 2, 128, 2048, False, False, True, 5e6),
}


def weight_names(cfg: ModelConfig):
    """(name, shape, init) in the reference's export order (export_model.py:171-204)."""
    H, I, D = cfg.H, cfg.I, cfg.D
    nq, nkv = cfg.HQ * D, cfg.HKV * D
    out = []
    for l in range(cfg.L):
        p = "L%02d." % l
        out += [(p + "q_proj.weight_t", [H, nq], "w"), (p + "k_proj.weight_t", [H, nkv], "w"),
                (p + "v_proj.weight_t", [H, nkv], "w"), (p + "o_proj.weight_t", [nq, H], "w")]
        if cfg.bias:
            out += [(p + "q_proj.bias", [nq], "b"), (p + "k_proj.bias", [nkv], "b"),
                    (p + "v_proj.bias", [nkv], "b")]
        out += [(p + "gate_proj.weight_t", [H, I], "w"), (p + "up_proj.weight_t", [H, I], "w"),
                (p + "down_proj.weight_t", [I, H], "w"),
                (p + "input_layernorm.weight", [H], "n"),
                (p + "post_attention_layernorm.weight", [H], "n")]
        if cfg.qk_norm:
            out += [(p + "q_norm.weight", [D], "n"), (p + "k_norm.weight", [D], "n")]
    out += [("embed.weight", [cfg.V, H], "w"), ("lm_head.weight_t", [H, cfg.V], "lm"),
            ("final_norm.weight", [H], "n")]
    return out


def rope_table(max_pos: int, D: int, theta: float):
    """bf16 cos/sin [1,1,max_pos,D] exactly as export_model.py:70-77 builds them."""
    import torch
    inv = 1.0 / (torch.tensor(theta, dtype=torch.float64) **
                 (torch.arange(0, D, 2, dtype=torch.float64) / D))
    pos = torch.arange(max_pos, dtype=torch.float64)
    freqs = torch.outer(pos, inv)
    cos = torch.cat([freqs.cos(), freqs.cos()], dim=-1).to(torch.bfloat16)
    sin = torch.cat([freqs.sin(), freqs.sin()], dim=-1).to(torch.bfloat16)
    return cos.unsqueeze(0).unsqueeze(1), sin.unsqueeze(0).unsqueeze(1)


def make_ids(V: int, seq: int, seed: int):
    import torch
    gen = torch.Generator().manual_seed(seed)
    return torch.randint(0, V, (1, seq), generator=gen, dtype=torch.long)


def _bf16_bits_of(t) -> bytes:
    import torch
    return t.detach().cpu().contiguous().view(torch.int16).numpy().tobytes()


def synth_values(name: str, n: int, seed: int, std: float, mean: float = 0.0) -> np.ndarray:
    """bf16 bits of a synthetic tensor, from libkernrelay's host generator."""
    from . import _lib
    return _lib.synth_normal(name, seed, std, n, mean=mean)


def write_model(out_dir, cfg: ModelConfig, seq: int, seed: int = 1234, max_pos: int = 4096,
                materialize: bool = True, weight_std: float = 0.02, norm_std: float = 0.0,
                bias_std: float = 0.02) -> Path:
    """Write a model directory.  Norm weights are 1 (norm_std=0, as BASELINE asks) or
    1 + N(0, norm_std^2); biases N(0, bias_std^2); matmul weights N(0, weight_std^2)."""
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    manifest = {
        "config": {
            "arch": cfg.arch, "hidden_size": cfg.H, "intermediate_size": cfg.I,
            "num_hidden_layers": cfg.L, "num_attention_heads": cfg.HQ,
            "num_key_value_heads": cfg.HKV, "head_dim": cfg.D, "vocab_size": cfg.V,
            "rms_norm_eps": cfg.eps, "qk_norm": cfg.qk_norm, "attention_bias": cfg.bias,
            "tie_word_embeddings": cfg.tied, "rope_theta": cfg.theta, "hidden_act": "silu",
        },
        "tensors": {}, "seq": seq, "seed": seed, "max_pos": max_pos,
        "generator": "kernrelay_b200.model_gen (SplitMix64 Irwin-Hall(12), bf16)",
    }
    cursor = 0
    with open(out / "weights.bin", "wb") as f:
        def put_bits(name, shape, bits: bytes, source_shape=None):
            nonlocal cursor
            ent = {"offset": cursor, "bytes": len(bits), "dtype": "bfloat16", "shape": list(shape)}
            if source_shape is not None:
                ent["source_shape"] = list(source_shape)
            manifest["tensors"][name] = ent
            f.write(bits)
            cursor += len(bits)

        for name, shape, kind in weight_names(cfg):
            n = int(np.prod(shape))
            if kind == "lm":
                if cfg.tied:
                    # reference: lm_head.weight_t = embed.weight^T (export_model.py:197-198)
                    if materialize:
                        emb = synth_values("embed.weight", cfg.V * cfg.H, seed, weight_std)
                        bits = emb.reshape(cfg.V, cfg.H).T.copy().tobytes()
                        put_bits(name, shape, bits, source_shape=[cfg.V, cfg.H])
                    else:
                        manifest["tensors"][name] = {
                            "shape": shape, "dtype": "bfloat16", "source_shape": [cfg.V, cfg.H],
                            "synth": {"kind": "transpose_of", "of": "embed.weight"}}
                    continue
                std, mean = weight_std, 0.0
            elif kind == "w":
                std, mean = weight_std, 0.0
            elif kind == "b":
                std, mean = bias_std, 0.0
            else:  # norm weights
                std, mean = norm_std, 1.0
            if std == 0.0 and kind == "n":
                spec = {"kind": "const", "value": 1.0}
                if materialize or n <= 65536:
                    bits = np.full(n, 0x3F80, dtype=np.uint16).tobytes()
                    put_bits(name, shape, bits)
                else:
                    manifest["tensors"][name] = {"shape": shape, "dtype": "bfloat16", "synth": spec}
                continue
            if materialize:
                put_bits(name, shape, synth_values(name, n, seed, std, mean).tobytes())
            else:
                manifest["tensors"][name] = {
                    "shape": shape, "dtype": "bfloat16",
                    "synth": {"kind": "normal", "std": std, "mean": mean, "seed": seed}}
        cos, sin = rope_table(max_pos, cfg.D, cfg.theta)
        put_bits("rope.cos", list(cos.shape), _bf16_bits_of(cos))
        put_bits("rope.sin", list(sin.shape), _bf16_bits_of(sin))
    make_ids(cfg.V, seq, seed).numpy().tofile(out / "ids.bin")
    (out / "manifest.json").write_text(json.dumps(manifest, indent=1))
    return out


def config_with(name: str, **overrides) -> ModelConfig:
    return replace(CONFIGS[name], **overrides)


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--config", required=True, choices=sorted(CONFIGS))
    ap.add_argument("--out", required=True)
    ap.add_argument("--seq", type=int, default=2048)
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--max-pos", type=int, default=4096)
    ap.add_argument("--layers", type=int, default=None, help="override the layer count")
    ap.add_argument("--synthetic", action="store_true",
                    help="do not store large tensors; the loader synthesises them on the GPU")
    a = ap.parse_args()
    cfg = CONFIGS[a.config]
    if a.layers:
        cfg = replace(cfg, L=a.layers)
    p = write_model(a.out, cfg, a.seq, a.seed, a.max_pos, materialize=not a.synthetic)
    print(json.dumps({"out": str(p), "config": asdict(cfg)}))


if __name__ == "__main__":
    main()
