"""Banded RoPE attention kernels (include/atlas_swa.h) against a dense float64 torch
restatement of atlas_jax/model.py:117-133 (tests/swa_ref.py), forward (o, lse) and
VJP (dq, dk, dv).  bf16 operands: 2e-2 relative (Frobenius)."""
import pytest
import torch

import swa_ref as SR

pytestmark = pytest.mark.gpu


def rel(a, b):
    return float((a.double() - b).norm() / b.norm())


@pytest.mark.parametrize("B,T,H,W,rope", [(1, 300, 2, 64, True), (2, 256, 1, 200, True), (1, 130, 2, 0, True),
                                          (1, 200, 1, 1000, True), (1, 384, 2, 128, False), (1, 1, 1, 64, True)])
def test_swa_forward_backward(B, T, H, W, rope):
    from atlas_b200.swa import sliding_window_attention, swa_forward
    from atlas_b200 import device_status
    torch.manual_seed(T + W)
    q, k, v = (torch.randn(B, T, H, 64, device="cuda").to(torch.bfloat16) for _ in range(3))
    do = torch.randn(B, T, H, 64, device="cuda").to(torch.bfloat16)
    o, lse = swa_forward(q, k, v, W, rope)
    qq, kk, vv = (x.detach().clone().requires_grad_(True) for x in (q, k, v))
    out = sliding_window_attention(qq, kk, vv, W, rope)
    out.backward(do)
    torch.cuda.synchronize()
    device_status()
    r = [x.detach().cpu().double().requires_grad_(True) for x in (q, k, v)]
    o_ref, lse_ref = SR.attention(*r, W, rope)
    o_ref.backward(do.cpu().double())
    assert rel(o.cpu(), o_ref.detach()) < 2e-2
    assert (lse.cpu().double() - lse_ref.detach()).abs().max() < 2e-2
    assert torch.equal(out.detach(), o)
    for g, ref, n in ((qq.grad, r[0].grad, "dq"), (kk.grad, r[1].grad, "dk"), (vv.grad, r[2].grad, "dv")):
        if ref.norm() < 1e-9:  # window 0: every query sees itself only, so dq = 0 exactly
            assert g.float().abs().max() < 1e-4, n
        else:
            assert rel(g.cpu(), ref) < 2e-2, n


def test_swa_mag_shape_smoke():
    """The MAG config's attention shape (window 1024, 12 heads) at T = 4096: finite
    outputs and the first 256 rows against the dense reference."""
    from atlas_b200.swa import swa_forward
    torch.manual_seed(0)
    B, T, H, W = 1, 4096, 12, 1024
    q, k, v = (torch.randn(B, T, H, 64, device="cuda").to(torch.bfloat16) for _ in range(3))
    o, lse = swa_forward(q, k, v, W)
    assert torch.isfinite(o.float()).all() and torch.isfinite(lse).all()
    n = 1280  # rows up to 1280 see keys only from [0, 1280): a causal prefix
    o_ref, _ = SR.attention(*(x[:, :n].cpu().double() for x in (q, k, v)), W)
    assert rel(o[:, :n].cpu(), o_ref) < 2e-2
