"""CPU: the oracle is pinned to Hugging Face transformers (the reference's own oracle,
scripts/export_model.py:211-223) through the committed golden fixtures, and its
weight generator is pinned bit-for-bit to libkernrelay's host generator."""
import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

from kernrelay_b200 import model_gen
from oracle import qwen_ref

GOLDEN = Path(__file__).resolve().parent / "golden"


def _maxrel(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.mark.parametrize("name,std,mean,offset", [
    ("L00.q_proj.weight_t", 0.02, 0.0, 0),
    ("embed.weight", 0.02, 0.0, 123456789),
    ("L03.input_layernorm.weight", 0.1, 1.0, 7),
    ("L27.down_proj.weight_t", 0.02, 0.0, 2 ** 33 + 5),
])
def test_numpy_generator_matches_library(krlib, name, std, mean, offset):
    n = 50000
    lib_bits = krlib.synth_normal(name, 1234, std, n, offset=offset, mean=mean)
    np_bits = qwen_ref.synth_normal_np(name, 1234, std, n, offset=offset, mean=mean)
    assert np.array_equal(lib_bits, np_bits)
    f = qwen_ref.bf16_bits_to_f32(np_bits)
    assert abs(f.mean() - mean) < 5 * std / np.sqrt(n) + 1e-3
    assert abs(f.std() - std) < 0.02 * std + 1e-4


@pytest.fixture(scope="module", params=sorted(p.stem for p in GOLDEN.glob("*.npz")))
def golden_case(request, tmp_path_factory, krlib):
    name = request.param
    g = np.load(GOLDEN / f"{name}.npz")
    meta = json.loads(str(g["meta"]))
    d = model_gen.write_model(tmp_path_factory.mktemp(name) / "m",
                              model_gen.CONFIGS[meta["config"]], meta["seq"], seed=meta["seed"],
                              norm_std=meta["norm_std"])
    assert hashlib.sha256((d / "weights.bin").read_bytes()).hexdigest() == str(g["weights_sha256"])
    assert hashlib.sha256((d / "ids.bin").read_bytes()).hexdigest() == str(g["ids_sha256"])
    return name, g, d


def test_oracle_matches_hf_exactly_with_hf_rope(golden_case):
    """With HF's float32 rotary tables the restatement reproduces HF to fp32 noise."""
    name, g, d = golden_case
    m = qwen_ref.Model(d)
    out = qwen_ref.prefill(m, rope="hf")
    L = m.L
    for l in range(L - 1):
        assert _maxrel(out["hidden"][l].numpy(), g["hf_hidden"][l]) < 1e-5, (name, l)
    assert _maxrel(out["final_x"].numpy(), g["hf_hidden"][L - 1]) < 1e-5
    assert _maxrel(out["logits_last"], g["hf_logits_last"]) < 1e-5
    assert int(np.argmax(out["logits_last"])) == int(np.argmax(g["hf_logits_last"]))


def test_oracle_with_reference_bf16_rope_tables_close_to_hf(golden_case):
    """The reference runtime feeds bf16-rounded cos/sin tables (export_model.py:70-77);
    that changes results by far less than the 1e-2 parity bar."""
    name, g, d = golden_case
    m = qwen_ref.Model(d)
    out = qwen_ref.prefill(m, rope="table")
    for l in range(m.L - 1):
        assert _maxrel(out["hidden"][l].numpy(), g["hf_hidden"][l]) < 2e-3, (name, l)
    assert _maxrel(out["logits_last"], g["hf_logits_last"]) < 1e-2


@pytest.mark.parametrize("tp", [2, 4])
def test_tp_restatement_equals_unsharded(golden_case, tp):
    name, g, d = golden_case
    m = qwen_ref.Model(d)
    if m.I % tp:
        pytest.skip("I not divisible")
    a = qwen_ref.prefill(m, tp=1)
    b = qwen_ref.prefill(m, tp=tp)
    for l in range(m.L):
        assert _maxrel(b["hidden"][l].numpy(), a["hidden"][l].numpy()) < 1e-5
    assert _maxrel(b["logits_last"], a["logits_last"]) < 1e-5


def test_micro_dag_tiling_is_exact():
    """Row tiling of the config-2 micro-DAG changes nothing but the schedule."""
    import torch
    g = torch.Generator().manual_seed(0)
    k, S, K, H = 2, 256, 64, 128
    X = [torch.randn(S, K, generator=g) for _ in range(k)]
    W = [torch.randn(K, H, generator=g) * 0.02 for _ in range(k)]
    R = torch.randn(S, H, generator=g)
    gamma = torch.ones(H)
    h1, x1 = qwen_ref.micro_dag(X, W, R, gamma, 1e-6, tiles=1)
    h4, x4 = qwen_ref.micro_dag(X, W, R, gamma, 1e-6, tiles=4)
    assert torch.equal(h1, h4) and torch.equal(x1, x4)


def test_ids_follow_reference_generator(tmp_path):
    """ids.bin = torch.randint(0, V, (1,S), manual_seed(seed)) (export_model.py:206-210)."""
    import torch
    cfg = model_gen.config_with("tiny-qwen2", L=1)
    d = model_gen.write_model(tmp_path / "m", cfg, 32, seed=77, materialize=False)
    ids = np.fromfile(d / "ids.bin", dtype=np.int64)
    gen = torch.Generator().manual_seed(77)
    ref = torch.randint(0, cfg.V, (1, 32), generator=gen, dtype=torch.long).numpy()[0]
    assert np.array_equal(ids, ref)


def test_synthetic_and_materialized_dirs_agree(tmp_path):
    """A manifest with synth entries denotes exactly the tensors a materialized dir stores."""
    cfg = model_gen.config_with("tiny-qwen3", L=1, V=256)
    a = qwen_ref.Model(model_gen.write_model(tmp_path / "a", cfg, 32, materialize=True, norm_std=0.1))
    b = qwen_ref.Model(model_gen.write_model(tmp_path / "b", cfg, 32, materialize=False, norm_std=0.1))
    for name in a.tensors:
        assert np.array_equal(a._bits(name), b._bits(name)), name
