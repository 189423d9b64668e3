"""The layer-level drop-in: atlas_b200.memory_layer.AtlasMemoryLayer (signature of
atlas_jax/memory_layer.py:599, scan on the B200 kernels) against the same layer
written entirely in torch float64 (prologue and epilogue as in
memory_layer.py:606-633 / 720-725, scan from tests/torch_ref.py), forward and
parameter gradients.  Exact path: 1e-4 (parameter gradients: max(1e-4, 2x the error of
the same restatement in float32), since the float32 layer inputs to the scan carry
their rounding into long gradient sums); tensor path: 2e-2 (relative, Frobenius)."""
import numpy as np
import pytest
import torch

import torch_ref as TR

pytestmark = pytest.mark.gpu


def _reference(layer, x, state=None, dtype=torch.float64):
    """torch restatement of the whole layer with the module's weights (float64, or
    float32 to measure the reference's own float32 error)."""
    P = {n: p.detach().to(dtype).requires_grad_(True) for n, p in layer.named_parameters()}
    cfg = layer.config
    B, T, C = x.shape
    H, D, E = layer.n_head, layer.head_dim, layer.expand_dim
    xd = x.to(dtype)

    def conv(name, z):
        zt = torch.nn.functional.pad(z.transpose(1, 2), (cfg.conv_kernel - 1, 0))
        return torch.nn.functional.conv1d(zt, P[f"{name}.weight"], P[f"{name}.bias"], groups=z.shape[-1]).transpose(1, 2)

    def rms(z):
        return z * torch.rsqrt((z * z).mean(-1, keepdim=True) + 1e-6)

    def poly(z):
        out, zp = P["poly_coeffs"][0] * z, z
        for i in range(1, cfg.poly_degree):
            zp = zp * z
            out = out + P["poly_coeffs"][i] * zp
        return out
    q = conv("conv_q", xd @ P["c_q.weight"].T).reshape(B, T, H, D)
    k = conv("conv_k", xd @ P["c_k.weight"].T).reshape(B, T, H, D)
    v = conv("conv_v", xd @ P["c_v.weight"].T).reshape(B, T, H, D)
    q, k = poly(rms(q)), rms(poly(k))
    gate = lambda n: torch.sigmoid(xd @ P[f"{n}.weight"].T + P[f"{n}.bias"])  # noqa: E731
    a, e, t, g = gate("gate_alpha"), gate("gate_eta") * cfg.max_lr, gate("gate_theta"), gate("gate_gamma")
    W1 = P["W1_init"].unsqueeze(0).expand(B, H, D, E)
    W2 = P["W2_init"].unsqueeze(0).expand(B, H, E, D)
    st = (W1, W2, torch.zeros_like(W1), torch.zeros_like(W2))
    y, _ = TR.scan(q, k, v, a, e, t, g, st, cfg.chunk_size, cfg.omega_window, cfg.ns_steps,
                   ste=cfg.pe_ste, stop_grad=cfg.stop_grad_chunks)
    y = y * torch.sigmoid(xd @ P["retrieve_gate.weight"].T).unsqueeze(-1)
    return y.reshape(B, T, H * D) @ P["c_proj.weight"].T, P


@pytest.mark.parametrize("prec,D,tol", [(0, 16, 1e-4), (1, 64, 2e-2)])
def test_memory_layer_forward_and_param_grads(prec, D, tol):
    from atlas_b200.memory_layer import AtlasConfig, AtlasMemoryLayer
    torch.manual_seed(0)
    H = 2
    cfg = AtlasConfig(n_embd=H * D, n_head=H, chunk_size=32, omega_window=8, memory_expand=4)
    layer = AtlasMemoryLayer(cfg, precision=prec).cuda()
    x = torch.randn(2, 45, H * D, device="cuda")
    y, state = layer(x)
    gy = torch.randn_like(y)
    (y * gy).sum().backward()
    y_ref, P = _reference(layer, x)
    (y_ref * gy.double()).sum().backward()
    rel = lambda a, b: float((a.double() - b.double()).norm() / b.double().norm())  # noqa: E731
    assert rel(y.detach(), y_ref.detach()) < tol
    if prec == 0:  # parameter gradients: within 2x the float32 restatement's own error
        y32, P32 = _reference(layer, x, dtype=torch.float32)
        (y32 * gy).sum().backward()
    for n, p in layer.named_parameters():
        if P[n].grad is None or P[n].grad.norm() == 0:
            continue
        bound = max(tol, 2.0 * rel(P32[n].grad, P[n].grad)) if prec == 0 else tol
        assert rel(p.grad, P[n].grad) < bound, (n, rel(p.grad, P[n].grad), bound)
    assert state.W1.shape == (2, H, D, 4 * D) and state.W2.shape == (2, H, 4 * D, D)
