"""krb_relay_down_single_noalloc (the allocation-free form of krb_relay_down_single)
called through the C ABI against the allocating entry point on the same inputs, and
against a plain torch fp32 computation of the same op (so a fault shared by both
entry points, which run the same kernel, cannot pass).

Named to be collected last, so it also runs after every other test of the
session; it passes alone in a fresh process as well, where its first call does
the per-device set-up.  Tolerance: the relay test's own bound (sum: 1e-3 * max|ref|
+ 1e-2; x: 1e-2 * max|ref|)."""
import pytest


def _close(got, ref, rel, abs_):
    got = got.float()
    ref = ref.float()
    err = (got - ref).abs().max().item()
    bound = rel * ref.abs().max().item() + abs_
    assert err <= bound, f"max abs err {err:.4g} > {bound:.4g}"


@pytest.mark.gpu
@pytest.mark.parametrize("S,H,K,tiles,bn", [(512, 896, 512, 4, 256),
                                            (1024, 3584, 2368, 4, 224)])
def test_noalloc_matches_allocating_entry(cuda, krlib, S, H, K, tiles, bn):
    import torch
    g = torch.Generator().manual_seed(S + H + 11)
    act = torch.randn(S, K, generator=g).to(torch.bfloat16).to(cuda)
    W = (torch.randn(H, K, generator=g) * 0.02).to(torch.bfloat16).to(cuda)
    resid = torch.randn(S, H, generator=g).to(cuda)
    gamma = (1 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16).to(cuda)

    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    s_ref, x_ref = krlib.relay_down_single(act, W, resid, gamma, tiles, 1e-6, bn=bn, status=status)
    torch.cuda.synchronize()
    assert status.item() == 0
    # independent fp32 reference: sum = resid + act . W^T, x = RMSNorm(sum) * gamma
    s_t = resid + act.float() @ W.float().T
    x_t = s_t * torch.rsqrt(s_t.pow(2).mean(-1, keepdim=True) + 1e-6) * gamma.float()

    # two calls in a row on one stream, each into fresh NaN-filled outputs, so a
    # call that skipped work (stale counters, wrong epoch) cannot pass
    for _ in range(2):
        st = torch.zeros(1, dtype=torch.int32, device=cuda)
        out = (torch.full((S, H), float("nan"), dtype=torch.float32, device=cuda),
               torch.full((S, H), float("nan"), dtype=torch.bfloat16, device=cuda))
        s, x = krlib.relay_down_single_noalloc(act, W, resid, gamma, tiles, 1e-6, bn=bn,
                                               status=st, out=out)
        torch.cuda.synchronize()
        assert st.item() == 0
        assert torch.isfinite(s).all() and torch.isfinite(x.float()).all()
        _close(s, s_ref, rel=1e-3, abs_=1e-2)
        _close(x, x_ref, rel=1e-2, abs_=0)
        _close(s, s_t, rel=1e-3, abs_=1e-2)
        _close(x, x_t, rel=1e-2, abs_=0)


def test_noalloc_rejects_tiles_beyond_scratch(krlib):
    """128 row tiles need (2*128+2)*128 = 33024 bytes: above the 32 KiB static
    scratch (127 tiles fill it exactly), rejected before any CUDA call (so this
    runs without a GPU)."""
    S = 128 * 128
    rc = krlib.lib().krb_relay_down_single_noalloc(None, None, None, None, None, None, S, 896,
                                                   512, 128, 1e-6, 256, None, None)
    assert rc != 0
    assert "static scratch" in krlib.lib().krb_last_error().decode()
