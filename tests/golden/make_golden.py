"""Generate the golden fixtures that pin the CPU oracle to Hugging Face transformers.

The reference's numerical oracle is the HF model run eagerly (scripts/export_model.py:
211-223).  For each test-sized configuration this script
  1. writes a seeded random-init model directory (kernrelay_b200.model_gen,
     non-trivial norm weights so gamma indexing is exercised),
  2. loads the same weights into HF Qwen2ForCausalLM / Qwen3ForCausalLM in fp32
     (eager attention) and runs the prefill with output_hidden_states=True,
  3. stores HF's per-layer hidden states and last-row logits, plus the sha256 of
     weights.bin and ids.bin (so generator drift is caught), in <name>.npz.

Run from the repository root:  python tests/golden/make_golden.py
(transformers 5.5.0 / torch 2.11 produced the committed files.)
"""
from __future__ import annotations

import hashlib
import json
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from kernrelay_b200 import model_gen  # noqa: E402
from oracle import qwen_ref  # noqa: E402

CASES = {
    # name: (config, seq, norm_std)
    "tiny_qwen2_s64": ("tiny-qwen2", 64, 0.1),
    "tiny_qwen3_s48": ("tiny-qwen3", 48, 0.1),
    "small_qwen2_gqa7_s40": ("small-qwen2-gqa7", 40, 0.1),
    "small_qwen3_gqa4_s40": ("small-qwen3-gqa4", 40, 0.1),
}


def sha256(p: Path) -> str:
    return hashlib.sha256(p.read_bytes()).hexdigest()


def hf_model(m: qwen_ref.Model, cfg: model_gen.ModelConfig):
    from transformers import Qwen2Config, Qwen2ForCausalLM, Qwen3Config, Qwen3ForCausalLM
    common = dict(hidden_size=m.H, intermediate_size=m.I, num_hidden_layers=m.L,
                  num_attention_heads=m.HQ, num_key_value_heads=m.HKV, vocab_size=m.V,
                  rms_norm_eps=m.eps, rope_theta=m.theta, tie_word_embeddings=m.tied,
                  max_position_embeddings=4096, attention_dropout=0.0)
    if cfg.arch == "qwen3_vl":
        hc = Qwen3Config(head_dim=m.D, attention_bias=False, **common)
        model = Qwen3ForCausalLM(hc)
    else:
        hc = Qwen2Config(**common)
        model = Qwen2ForCausalLM(hc)
    model = model.float().eval()
    sd = {}
    sd["model.embed_tokens.weight"] = m.w("embed.weight")
    for l in range(m.L):
        p, q = "L%02d." % l, "model.layers.%d." % l
        for role in ("q_proj", "k_proj", "v_proj", "o_proj"):
            sd[q + "self_attn.%s.weight" % role] = m.w(p + role + ".weight_t").T.contiguous()
        if m.bias:
            for role in ("q_proj", "k_proj", "v_proj"):
                sd[q + "self_attn.%s.bias" % role] = m.w(p + role + ".bias")
        for role in ("gate_proj", "up_proj", "down_proj"):
            sd[q + "mlp.%s.weight" % role] = m.w(p + role + ".weight_t").T.contiguous()
        sd[q + "input_layernorm.weight"] = m.w(p + "input_layernorm.weight")
        sd[q + "post_attention_layernorm.weight"] = m.w(p + "post_attention_layernorm.weight")
        if m.qk_norm:
            sd[q + "self_attn.q_norm.weight"] = m.w(p + "q_norm.weight")
            sd[q + "self_attn.k_norm.weight"] = m.w(p + "k_norm.weight")
    sd["model.norm.weight"] = m.w("final_norm.weight")
    sd["lm_head.weight"] = m.w("lm_head.weight_t").T.contiguous()
    missing, unexpected = model.load_state_dict(sd, strict=False)
    missing = [k for k in missing if "rotary" not in k]
    if missing or unexpected:
        raise RuntimeError(f"state dict mismatch: missing={missing} unexpected={unexpected}")
    try:
        model.config._attn_implementation = "eager"
    except Exception:
        pass
    return model


def make(name: str, out_dir: Path):
    cfg_name, seq, norm_std = CASES[name]
    cfg = model_gen.CONFIGS[cfg_name]
    with tempfile.TemporaryDirectory() as td:
        d = model_gen.write_model(Path(td) / name, cfg, seq, seed=1234, norm_std=norm_std)
        m = qwen_ref.Model(d)
        model = hf_model(m, cfg)
        ids = torch.from_numpy(m.ids.copy())[None]
        with torch.no_grad():
            out = model(input_ids=ids, output_hidden_states=True)
        hs = [h[0].float().numpy() for h in out.hidden_states]
        np.savez_compressed(
            out_dir / f"{name}.npz",
            hf_hidden=np.stack(hs[1:]),                 # L entries: layers 0..L-2 residual, then normed final
            hf_logits_last=out.logits[0, -1].float().numpy(),
            weights_sha256=np.array(sha256(d / "weights.bin")),
            ids_sha256=np.array(sha256(d / "ids.bin")),
            meta=np.array(json.dumps({"config": cfg_name, "seq": seq, "norm_std": norm_std,
                                      "seed": 1234, "transformers": __import__("transformers").__version__,
                                      "torch": torch.__version__})),
        )
    print("wrote", out_dir / f"{name}.npz")


def main():
    names = sys.argv[1:] or list(CASES)
    for name in names:
        make(name, HERE)


if __name__ == "__main__":
    main()
