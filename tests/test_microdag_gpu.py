"""BASELINE configs[1], the isolated TP-MLP micro-DAG (mm -> AllReduce -> AddNorm with 4 row
tiles, qwen_main.cpp:1274-1302) at its exact shapes: per rank X_r [2048, 18944/k] ~ N(0,1),
W_r [18944/k, 3584] ~ N(0,0.02), residual R [2048, 3584] ~ N(0,1), gamma 1, eps 1e-6.

The fused relay (tp{k}_split) and the unfused GEMM + NCCL AllReduce baseline (tp{k}) are
compared with the oracle's micro_dag summing the k exact fp32 partials, through the
engine's C ABI.  The engine keeps the partials in fp32 at k = 1 and in fp16 at k > 1 (the
reference rounds them to bf16, qwen_main.cpp:1283-1287; fp16 rounds 8x finer).  Bar: h
within 1e-3 * max|h| + 1e-2 (fp16 rounding of up to k partials), x within 1e-2 * max|x|."""
import threading

import numpy as np
import pytest

from oracle import qwen_ref

pytestmark = pytest.mark.gpu

S, H, I, T, SEED = 2048, 3584, 18944, 4, 1234


def _ngpu():
    import torch
    return torch.cuda.device_count()


def _oracle(krlib, k):
    import torch
    K = I // k

    def t(name, seed, std, shape):
        bits = krlib.synth_normal(name, seed, std, int(np.prod(shape)))
        return torch.from_numpy(qwen_ref.bf16_bits_to_f32(bits).reshape(shape))
    X = [t("microdag.X", SEED + r, 1.0, (S, K)) for r in range(k)]
    W = [t("microdag.W_down", SEED + r, 0.02, (K, H)) for r in range(k)]
    R = t("microdag.R", SEED, 1.0, (S, H))
    h, x = qwen_ref.micro_dag(X, W, R, torch.ones(H), 1e-6, tiles=T, round_partials=False)
    return h.numpy(), x.numpy()


def _check(eng, h_ref, x_ref, label):
    h = eng.final_hidden()
    x = eng.final_x()
    eh = float(np.abs(h - h_ref).max())
    ex = float(np.abs(x - x_ref).max())
    print(f"\n{label}: h max abs err {eh:.3e} (max|h| {np.abs(h_ref).max():.3g}), "
          f"x max abs err {ex:.3e} (max|x| {np.abs(x_ref).max():.3g})")
    assert eh <= 1e-3 * np.abs(h_ref).max() + 1e-2, f"{label}: h max abs err {eh:.4g}"
    assert ex <= 1e-2 * np.abs(x_ref).max(), f"{label}: x max abs err {ex:.4g}"


@pytest.fixture(scope="module")
def ref1(krlib):
    return _oracle(krlib, 1)


@pytest.mark.parametrize("mode", ["tp1_split", "tp1"])
def test_microdag_k1_matches_oracle(cuda, krlib, ref1, mode):
    eng = krlib.Engine.microdag(S, H, I, mode, tiles=T, seed=SEED)
    try:
        eng.capture()
        for _ in range(2):   # graph replays: epochs advance, counters stay monotone
            eng.run()
        eng.sync()
        assert eng.status() == 0
        _check(eng, *ref1, mode)
    finally:
        eng.close()


@pytest.mark.multigpu
@pytest.mark.parametrize("k", [2, 4, 8])
@pytest.mark.parametrize("variant", ["split", "nccl"])
def test_microdag_multi_gpu_matches_oracle(cuda, krlib, k, variant):
    """k ranks in one process (one host thread each): every rank's h and x against the
    oracle's sum of the k ranks' bf16 partials."""
    if _ngpu() < k:
        pytest.skip(f"needs {k} GPUs")
    mode = f"tp{k}_split" if variant == "split" else f"tp{k}"
    h_ref, x_ref = _oracle(krlib, k)
    engines = [krlib.Engine.microdag(S, H, I, mode, rank=r, world=k, device=r, tiles=T, seed=SEED)
               for r in range(k)]
    try:
        if variant == "split":
            krlib.Engine.link(engines)
        else:
            krlib.Engine.init_nccl_all(engines)
        errs = []

        def go(e):
            try:
                for _ in range(3):
                    e.run()
                e.sync()
            except Exception as ex:  # noqa: BLE001
                errs.append(ex)
        th = [threading.Thread(target=go, args=(e,)) for e in engines]
        for t in th:
            t.start()
        for t in th:
            t.join()
        if errs:
            raise errs[0]
        for e in engines:
            assert e.status() == 0, f"rank {e.rank}: status {e.status()}"
            _check(e, h_ref, x_ref, f"{mode} rank {e.rank}")
    finally:
        for e in engines:
            e.close()
