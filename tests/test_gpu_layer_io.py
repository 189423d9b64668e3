"""Fused layer prologue / retrieve gate (include/atlas_layer.h) against the oracle's
numpy restatement (forward) and torch float64 autograd of the same math (VJP).
Reference: atlas_jax/memory_layer.py:606-633, 720-722.  Tolerances: float32 1e-5
(forward) / 1e-4 (VJP), relative Frobenius; bf16 activations 1e-2 (one output rounding)."""
import numpy as np
import pytest
import torch

import layer_ref as LR
from oracle import atlas_oracle as O

pytestmark = pytest.mark.gpu

CASES = [  # B, T, H, D, K, poly_degree, gamma, retrieve, padded rows (16-byte lanes)
    (2, 70, 3, 64, 4, 2, True, True, True),
    (2, 70, 3, 64, 4, 2, True, True, False),   # unpadded rows: the per-channel kernels
    (1, 1, 2, 32, 4, 2, True, True, True),     # T < K
    (2, 33, 1, 16, 3, 0, False, False, True),  # no poly, no gamma / retrieve, D < 32
    (1, 40, 2, 128, 4, 3, False, True, True),
    (1, 17, 2, 256, 8, 1, True, False, True),
    (1, 9, 3, 48, 4, 2, True, True, True),     # D / 8 does not divide 32: per-channel kernels
]


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _setup(case, dtype, seed=0):
    from atlas_b200.layer_io import LayerGeometry
    B, T, H, D, K, P, hg, hr, pad = case
    geo = LayerGeometry(B, T, H, D, K, P, hg, hr, 0.1, pad)
    rng = np.random.default_rng(seed)
    proj = rng.standard_normal((B * T, geo.proj_stride)).astype(np.float32)
    cw, cb, poly, gb = LR.make_params(H, D, K, P, geo.n_gates - int(hr), seed)
    tproj = torch.as_tensor(proj).cuda().to(dtype)
    proj = tproj.float().cpu().numpy()  # what the kernel sees
    dev = lambda x: None if x is None else torch.as_tensor(x).cuda()  # noqa: E731
    cw_k = np.ascontiguousarray(cw.transpose(0, 2, 1))  # the kernel's tap-major layout (3, K, H*D)
    return geo, proj, (cw, cb, poly, gb), tproj, [dev(x) for x in (cw_k, cb, poly, gb)]


@pytest.mark.parametrize("case", CASES)
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_prologue_forward(case, dtype):
    from atlas_b200.layer_io import prologue_forward
    geo, proj, (cw, cb, poly, gb), tproj, dp = _setup(case, dtype)
    q, k, v, g = prologue_forward(geo, tproj, *dp)
    qo, ko, vo, go = O.layer_prologue(proj[:, :geo.n_proj].astype(np.float64), geo.B, geo.T, geo.H, geo.D, cw, cb, poly, gb,
                                      geo.has_gamma, geo.has_retrieve, geo.max_lr)
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    for a, b in ((q, qo), (k, ko), (v, vo)):
        assert rel(a.float().cpu().numpy(), b) < tol
    for a, b in zip(g, go):
        assert (a is None) == (b is None)
        if a is not None:
            assert rel(a.cpu().numpy(), b) < 1e-5


@pytest.mark.parametrize("case", CASES)
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_prologue_backward(case, dtype):
    from atlas_b200.layer_io import prologue_backward
    geo, proj, (cw, cb, poly, gb), tproj, dp = _setup(case, dtype, seed=3)
    rng = np.random.default_rng(7)
    B, T, H, D = geo.B, geo.T, geo.H, geo.D
    dq, dk, dv = (rng.standard_normal((B, T, H, D)).astype(np.float32) for _ in range(3))
    dgs = [rng.standard_normal((B, T, H)).astype(np.float32) for _ in range(5)]
    if not geo.has_gamma:
        dgs[3] = None
    if not geo.has_retrieve:
        dgs[4] = None
    cu = lambda x, dt=torch.float32: None if x is None else torch.as_tensor(x).cuda().to(dt)  # noqa: E731
    dproj, dcw, dcb, dpoly, dgb = prologue_backward(geo, tproj, *dp, cu(dq, dtype), cu(dk, dtype), cu(dv, dtype),
                                                    [cu(x) for x in dgs])
    # float64 autograd of the restatement, with the cotangents as the kernel saw them
    leaf = lambda x: None if x is None else torch.tensor(x, dtype=torch.float64, requires_grad=True)  # noqa: E731
    proj = proj[:, :geo.n_proj]
    P_, cw_, cb_, poly_, gb_ = leaf(proj), leaf(cw), leaf(cb), leaf(poly), leaf(gb)
    q, k, v, g = LR.prologue(P_, B, T, H, D, cw_, cb_, poly_, gb_, geo.has_gamma, geo.has_retrieve, geo.max_lr)
    as64 = lambda x, dt: torch.as_tensor(x).to(dt).double()  # noqa: E731
    loss = sum((o * as64(c, dtype)).sum() for o, c in ((q, dq), (k, dk), (v, dv)))
    loss = loss + sum((o * torch.as_tensor(c).double()).sum() for o, c in zip(g, dgs) if o is not None)
    loss.backward()
    tol = 1e-4 if dtype == torch.float32 else 1e-2
    assert rel(dproj[:, :geo.n_proj].float().cpu().numpy(), P_.grad.numpy()) < tol
    assert float(dproj[:, geo.n_proj:].float().abs().max()) == 0.0 if geo.proj_stride > geo.n_proj else True
    assert rel(dcw.cpu().numpy().transpose(0, 2, 1), cw_.grad.numpy()) < tol
    assert rel(dcb.cpu().numpy(), cb_.grad.numpy()) < tol
    assert rel(dgb.cpu().numpy(), gb_.grad.numpy()) < tol
    if poly is not None:
        assert rel(dpoly.cpu().numpy(), poly_.grad.numpy()) < tol


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_retrieve_gate(dtype):
    from atlas_b200.layer_io import LayerGeometry, retrieve_gate
    B, T, H, D = 2, 37, 3, 64
    geo = LayerGeometry(B, T, H, D)
    torch.manual_seed(0)
    y = torch.randn(B, T, H, D, device="cuda").to(dtype).requires_grad_(True)
    r = torch.rand(B, T, H, device="cuda").requires_grad_(True)
    yg = retrieve_gate(geo, y, r)
    gy = torch.randn_like(yg)
    (yg.float() * gy.float()).sum().backward()
    yd, rd = y.detach().double().requires_grad_(True), r.detach().double().requires_grad_(True)
    ref = yd * rd.unsqueeze(-1)
    (ref * gy.double()).sum().backward()
    tol = 1e-6 if dtype == torch.float32 else 1e-2
    assert rel(yg.detach().float().cpu(), ref.detach().cpu()) < tol
    assert rel(y.grad.float().cpu(), yd.grad.cpu()) < tol
    assert rel(r.grad.cpu(), rd.grad.cpu()) < max(tol, 1e-5)
