"""Each hot-path kernel, called through the C ABI, against a plain PyTorch fp32
statement of the same op on the same seeded inputs.

Tolerances: outputs are bf16, so one output rounding is 2^-8 relative; GEMMs
accumulate in fp32 (different order than torch), so errors are bounded by
|err| <= 1e-2 * max|ref| + 1e-2 (stated per test)."""
import math

import pytest

pytestmark = pytest.mark.gpu


def _close(got, ref, rel=1e-2, abs_=1e-2):
    got = got.float()
    ref = ref.float()
    err = (got - ref).abs().max().item()
    bound = rel * ref.abs().max().item() + abs_
    assert err <= bound, f"max abs err {err:.4g} > {bound:.4g}"


def _bf(t):
    import torch
    return t.to(torch.bfloat16).contiguous()


@pytest.mark.parametrize("M,N,K,bn", [
    (256, 512, 512, 256),
    (256, 448, 640, 224),
    (384, 256, 1024, 128),
    (200, 136, 96, 128),     # ragged M, N, and K not a multiple of 64
    (128, 896, 896, 256),    # 0.5B hidden: last N block half full
    (512, 3584, 2368, 0),    # 7B down at k=8 (K = 37 * 64), automatic tile
])
def test_gemm(cuda, krlib, M, N, K, bn):
    import torch
    g = torch.Generator(device="cpu").manual_seed(M * 7 + N + K)
    A = _bf(torch.randn(M, K, generator=g)).to(cuda)
    B = _bf(torch.randn(N, K, generator=g) * 0.05).to(cuda)
    C = krlib.gemm(A, B, bn=bn)
    torch.cuda.synchronize()
    ref = A.float() @ B.float().T
    _close(C, ref)


@pytest.mark.parametrize("M,N,K,bn", [(256, 3584, 512, 224), (200, 896, 640, 256),
                                      (384, 512, 2368, 128)])
def test_gemm_f32_output(cuda, krlib, M, N, K, bn):
    import torch
    g = torch.Generator().manual_seed(M + N)
    A = _bf(torch.randn(M, K, generator=g)).to(cuda)
    B = _bf(torch.randn(N, K, generator=g) * 0.05).to(cuda)
    C = krlib.gemm_f32(A, B, bn=bn)
    torch.cuda.synchronize()
    ref = A.float() @ B.float().T
    # fp32 accumulate, no output rounding: far tighter than the bf16-output bound
    _close(C, ref, rel=1e-4, abs_=1e-4)


def test_gemm_bias_and_pitch(cuda, krlib):
    import torch
    g = torch.Generator().manual_seed(3)
    M, N, K = 256, 384, 512
    A = _bf(torch.randn(M, K, generator=g)).to(cuda)
    B = _bf(torch.randn(N, K, generator=g) * 0.05).to(cuda)
    bias = _bf(torch.randn(N, generator=g)).to(cuda)
    big = torch.zeros(M, N + 64, dtype=torch.bfloat16, device=cuda)
    out = big[:, 32:32 + N]
    krlib.gemm(A, B, bias=bias, out=out, bn=128)
    torch.cuda.synchronize()
    _close(out, A.float() @ B.float().T + bias.float())
    assert big[:, :32].abs().max().item() == 0 and big[:, 32 + N:].abs().max().item() == 0


@pytest.mark.parametrize("M,I,K,bn", [(256, 512, 512, 256), (256, 320, 384, 128),
                                      (512, 2368, 896, 256), (512, 2368, 896, 192),
                                      (384, 1216, 640, 192)])
def test_gemm_silu(cuda, krlib, M, I, K, bn):
    """bn 192: the 7B / Qwen3-VL-4B tp8 gate/up widths (2368, 1216 per rank); M = 384 has
    an odd number of 128-row blocks, so it runs on one-CTA tiles instead of CTA pairs."""
    import torch
    g = torch.Generator().manual_seed(I + K)
    A = _bf(torch.randn(M, K, generator=g)).to(cuda)
    Wg = _bf(torch.randn(I, K, generator=g) * 0.05).to(cuda)
    Wu = _bf(torch.randn(I, K, generator=g) * 0.05).to(cuda)
    Bgu = krlib.interleave_gate_up(Wg, Wu, bn)
    act = krlib.gemm_silu(A, Bgu, I, bn)
    torch.cuda.synchronize()
    gate = A.float() @ Wg.float().T
    up = A.float() @ Wu.float().T
    ref = torch.nn.functional.silu(gate) * up
    _close(act, ref)


@pytest.mark.parametrize("rows,H", [(64, 896), (33, 3584), (16, 4096), (8, 8192)])
def test_rmsnorm(cuda, krlib, rows, H):
    import torch
    g = torch.Generator().manual_seed(rows + H)
    x = _bf(torch.randn(rows, H, generator=g)).to(cuda)
    gamma = _bf(1 + 0.1 * torch.randn(H, generator=g)).to(cuda)
    y = krlib.rmsnorm(x, gamma, 1e-6)
    torch.cuda.synchronize()
    xf = x.float()
    ref = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * gamma.float()
    _close(y, ref, rel=1e-2, abs_=0)


def test_add_rmsnorm(cuda, krlib):
    import torch
    g = torch.Generator().manual_seed(5)
    rows, H = 96, 3584
    a = _bf(torch.randn(rows, H, generator=g)).to(cuda)
    b = _bf(torch.randn(rows, H, generator=g)).to(cuda)
    gamma = _bf(1 + 0.1 * torch.randn(H, generator=g)).to(cuda)
    y, s = krlib.add_rmsnorm(a, b, gamma, 1e-6)
    torch.cuda.synchronize()
    sref = (a.float() + b.float()).to(torch.bfloat16)
    assert torch.equal(s, sref)
    sf = sref.float()
    ref = sf * torch.rsqrt(sf.pow(2).mean(-1, keepdim=True) + 1e-6) * gamma.float()
    _close(y, ref, rel=1e-2, abs_=0)


def test_add_rmsnorm_fp32_residual(cuda, krlib):
    import torch
    g = torch.Generator().manual_seed(6)
    rows, H = 80, 2560
    res = torch.randn(rows, H, generator=g).to(cuda)
    delta = _bf(torch.randn(rows, H, generator=g)).to(cuda)
    gamma = _bf(1 + 0.1 * torch.randn(H, generator=g)).to(cuda)
    y, s = krlib.add_rmsnorm_res(res, delta, gamma, 1e-6)
    torch.cuda.synchronize()
    sref = res + delta.float()
    assert (s - sref).abs().max().item() <= 1e-6 * sref.abs().max().item()
    ref = sref * torch.rsqrt(sref.pow(2).mean(-1, keepdim=True) + 1e-6) * gamma.float()
    _close(y, ref, rel=1e-2, abs_=0)


def test_embed(cuda, krlib):
    import torch
    g = torch.Generator().manual_seed(9)
    V, H, S = 1000, 896, 77
    table = _bf(torch.randn(V, H, generator=g)).to(cuda)
    ids = torch.randint(0, V, (S,), generator=g).to(cuda)
    out = krlib.embed(ids, table)
    torch.cuda.synchronize()
    assert torch.equal(out, table[ids])


def test_embed_out_of_range_sets_status(cuda, krlib):
    import torch
    V, H = 64, 128
    table = torch.ones(V, H, dtype=torch.bfloat16, device=cuda)
    ids = torch.tensor([1, V + 5, -1, 3], device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = krlib.embed(ids, table, status=status)
    torch.cuda.synchronize()
    assert status.item() & (1 << 7)
    assert out[1].abs().max().item() == 0 and out[2].abs().max().item() == 0
    assert out[0].float().min().item() == 1.0


def _rope_ref(x, cos, sin):
    # x [S, h, D] fp32; rotate-half
    D = x.shape[-1]
    x1, x2 = x[..., : D // 2], x[..., D // 2:]
    rot = torch_cat(-x2, x1)
    return x * cos[:, None, :] + rot * sin[:, None, :]


def torch_cat(a, b):
    import torch
    return torch.cat([a, b], dim=-1)


def _rope_tables(S, D, theta):
    import torch
    inv = 1.0 / (torch.tensor(theta, dtype=torch.float64) **
                 (torch.arange(0, D, 2, dtype=torch.float64) / D))
    f = torch.outer(torch.arange(S, dtype=torch.float64), inv)
    cos = torch.cat([f.cos(), f.cos()], -1).to(torch.bfloat16)
    sin = torch.cat([f.sin(), f.sin()], -1).to(torch.bfloat16)
    return cos, sin


@pytest.mark.parametrize("S,HQ,HKV,D,qk_norm,bias", [(256, 4, 2, 128, True, False),
                                                     (200, 6, 2, 64, False, True),
                                                     (384, 28, 4, 128, False, True)])
def test_gemm_qkv_rope(cuda, krlib, S, HQ, HKV, D, qk_norm, bias):
    """Fused QKV GEMM + bias + QK-norm + RoPE epilogue vs torch fp32 of the same op
    (GEMM in fp32; the normalised q/k rounded to bf16 as in the kernel)."""
    import torch
    g = torch.Generator().manual_seed(S + D)
    H = 512
    N = (HQ + 2 * HKV) * D
    A = _bf(torch.randn(S, H, generator=g)).to(cuda)
    B = _bf(torch.randn(N, H, generator=g) * 0.05).to(cuda)
    b = _bf(torch.randn(N, generator=g) * 0.1).to(cuda) if bias else None
    cos, sin = _rope_tables(S, D, 1e6)
    cos, sin = cos.to(cuda), sin.to(cuda)
    qn = _bf(1 + 0.1 * torch.randn(D, generator=g)).to(cuda) if qk_norm else None
    kn = _bf(1 + 0.1 * torch.randn(D, generator=g)).to(cuda) if qk_norm else None
    ldvt = (S + 7) // 8 * 8
    vt = torch.full((HKV * D, ldvt), float("nan"), dtype=torch.float16, device=cuda)
    out = krlib.gemm_qkv_rope(A, B, HQ, HKV, D, cos, sin, bias=b, q_norm=qn, k_norm=kn, vt=vt)
    torch.cuda.synchronize()
    # the transposed v heads are exactly the stored bf16 v columns, in fp16
    v_cols = out[:, (HQ + HKV) * D:]
    assert torch.equal(vt[:, :S], v_cols.float().half().T)
    x = A.float() @ B.float().T
    if b is not None:
        x = x + b.float()
    x = x.view(S, HQ + 2 * HKV, D)
    q, k, v = x[:, :HQ], x[:, HQ:HQ + HKV], x[:, HQ + HKV:]
    if qk_norm:
        q = (q * torch.rsqrt(q.pow(2).mean(-1, keepdim=True) + 1e-6) * qn.float()).to(torch.bfloat16).float()
        k = (k * torch.rsqrt(k.pow(2).mean(-1, keepdim=True) + 1e-6) * kn.float()).to(torch.bfloat16).float()
    qr = _rope_ref(q, cos.float(), sin.float())
    kr = _rope_ref(k, cos.float(), sin.float())
    ref = torch.cat([qr, kr, v], 1).reshape(S, N)
    _close(out, ref, rel=1e-2, abs_=2e-2)


@pytest.mark.parametrize("D,qk_norm", [(64, False), (128, True), (128, False)])
def test_qk_norm_rope(cuda, krlib, D, qk_norm):
    import torch
    g = torch.Generator().manual_seed(D)
    S, HQ, HKV = 100, 4, 2
    qkv = _bf(torch.randn(S, (HQ + 2 * HKV) * D, generator=g)).to(cuda)
    cos, sin = _rope_tables(S, D, 1e6)
    cos, sin = cos.to(cuda), sin.to(cuda)
    qn = _bf(1 + 0.1 * torch.randn(D, generator=g)).to(cuda) if qk_norm else None
    kn = _bf(1 + 0.1 * torch.randn(D, generator=g)).to(cuda) if qk_norm else None
    orig = qkv.clone()
    krlib.qk_norm_rope(qkv, HQ, HKV, D, cos, sin, qn, kn, 1e-6)
    torch.cuda.synchronize()
    x = orig.float().view(S, HQ + 2 * HKV, D)
    q, k, v = x[:, :HQ], x[:, HQ:HQ + HKV], x[:, HQ + HKV:]
    if qk_norm:
        q = (q * torch.rsqrt(q.pow(2).mean(-1, keepdim=True) + 1e-6) * qn.float()).to(torch.bfloat16).float()
        k = (k * torch.rsqrt(k.pow(2).mean(-1, keepdim=True) + 1e-6) * kn.float()).to(torch.bfloat16).float()
    qr = _rope_ref(q, cos.float(), sin.float())
    kr = _rope_ref(k, cos.float(), sin.float())
    got = qkv.float().view(S, HQ + 2 * HKV, D)
    _close(got[:, :HQ], qr, rel=1e-2, abs_=0)
    _close(got[:, HQ:HQ + HKV], kr, rel=1e-2, abs_=0)
    assert torch.equal(got[:, HQ + HKV:], v)  # v untouched


def _attn_ref(qkv, S, HQ, HKV, D, scale):
    import torch
    x = qkv.float().view(S, HQ + 2 * HKV, D)
    q, k, v = x[:, :HQ], x[:, HQ:HQ + HKV], x[:, HQ + HKV:]
    rep = HQ // HKV
    k = k.repeat_interleave(rep, dim=1)
    v = v.repeat_interleave(rep, dim=1)
    s = torch.einsum("qhd,khd->hqk", q, k) * scale
    mask = torch.triu(torch.ones(S, S, dtype=torch.bool, device=qkv.device), 1)
    s = s.masked_fill(mask, float("-inf"))
    p = torch.softmax(s, -1)
    return torch.einsum("hqk,khd->qhd", p, v).reshape(S, HQ * D)


@pytest.mark.parametrize("S,HQ,HKV,D,impl", [
    # tcgen05/TMEM kernel: multiples of the 128-row tile, ragged S, GQA groups, MHA,
    # head_dim 64 (Qwen2.5-0.5B: 14 / 2 heads) and 128
    (128, 4, 2, 64, 2), (70, 2, 2, 64, 0), (512, 14, 2, 64, 2), (1000, 4, 1, 64, 2),
    (128, 2, 1, 128, 2), (512, 8, 2, 128, 2), (200, 4, 1, 128, 2), (1000, 4, 4, 128, 2),
    (2048, 28, 4, 128, 2),
])
def test_attention(cuda, krlib, S, HQ, HKV, D, impl):
    import torch
    g = torch.Generator().manual_seed(S + D + impl)
    qkv = _bf(torch.randn(S, (HQ + 2 * HKV) * D, generator=g)).to(cuda)
    scale = 1.0 / math.sqrt(D)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = krlib.attention(qkv, HQ, HKV, D, scale, impl=impl, status=status)
    torch.cuda.synchronize()
    assert status.item() == 0
    ref = _attn_ref(qkv, S, HQ, HKV, D, scale)
    _close(out, ref, rel=2e-2, abs_=1e-2)


@pytest.mark.parametrize("S,H,K,tiles,bn", [(512, 896, 512, 4, 256), (256, 384, 256, 2, 128),
                                            (1024, 3584, 2368, 4, 224)])
def test_relay_down_single(cuda, krlib, S, H, K, tiles, bn):
    """Fused down GEMM + tile relay + Add+RMSNorm (one device) vs torch fp32."""
    import torch
    g = torch.Generator().manual_seed(S + H)
    act = _bf(torch.randn(S, K, generator=g)).to(cuda)
    W = _bf(torch.randn(H, K, generator=g) * 0.02).to(cuda)
    resid = torch.randn(S, H, generator=g).to(cuda)
    gamma = _bf(1 + 0.1 * torch.randn(H, generator=g)).to(cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    s, x = krlib.relay_down_single(act, W, resid, gamma, tiles, 1e-6, bn=bn, status=status)
    torch.cuda.synchronize()
    assert status.item() == 0
    down = (act.float() @ W.float().T).to(torch.bfloat16).float()
    sref = resid + down
    _close(s, sref, rel=1e-3, abs_=1e-2)
    sf = s.float()
    xref = sf * torch.rsqrt(sf.pow(2).mean(-1, keepdim=True) + 1e-6) * gamma.float()
    _close(x, xref, rel=1e-2, abs_=0)
