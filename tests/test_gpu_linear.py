"""Linear-memory variant (atlas_jax/memory_layer.py:468-494) on the float64 path:
forward against the oracle, backward against torch float64 autograd of
tests/torch_ref.scan_linear (whose forward is checked against the oracle on CPU).
float32 activations: 1e-5 relative; bf16 activations: 2e-2."""
import numpy as np
import pytest
import torch

import torch_ref as TR
from oracle import atlas_oracle as O

pytestmark = pytest.mark.gpu


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


CASES = [  # B, T, H, D, chunk, omega, state, stop_grad
    (2, 45, 2, 16, 16, 4, True, False),
    (1, 64, 2, 32, 32, 1, False, False),
    (1, 33, 1, 16, 8, 16, True, True),   # omega >= chunk, detached carries
    (1, 1, 1, 32, 16, 4, True, False),   # a single token
]


@pytest.mark.parametrize("case", CASES)
@pytest.mark.parametrize("act", [torch.float32, torch.bfloat16])
def test_linear_exact_forward_backward(case, act):
    from atlas_b200 import ATLAS_PREC_EXACT, ScanConfig, device_status, linear_scan_backward, linear_scan_forward
    B, T, H, D, cs, om, has_state, sg = case
    ins = list(O.make_inputs(B, T, H, D, seed=T + D, gamma_mode="random"))
    if act == torch.bfloat16:  # the inputs as the kernel sees them
        ins[:3] = [torch.as_tensor(x).to(act).float().numpy() for x in ins[:3]]
    rng = np.random.default_rng(5)
    st = (0.1 * rng.standard_normal((B, H, D, D)).astype(np.float32),
          0.01 * rng.standard_normal((B, H, D, D)).astype(np.float32)) if has_state else None
    dy = rng.standard_normal((B, T, H, D)).astype(np.float32)
    if act == torch.bfloat16:
        dy = torch.as_tensor(dy).to(act).float().numpy()
    dM = rng.standard_normal((B, H, D, D)).astype(np.float32) * 0.1
    cfg = ScanConfig(chunk=cs, omega=om, ns_steps=5, stop_grad_chunks=sg, precision=ATLAS_PREC_EXACT)
    cu = lambda x, dt=torch.float32: None if x is None else torch.as_tensor(x).cuda().to(dt)  # noqa: E731
    dins = [cu(x, act) for x in ins[:3]] + [cu(x) for x in ins[3:]]
    dst = None if st is None else tuple(cu(x) for x in st)
    y, out = linear_scan_forward(*dins, dst, cfg)
    grads = linear_scan_backward(*dins, dst, cu(dy, act), (cu(dM), None), cfg)
    torch.cuda.synchronize()
    device_status()
    tol = 1e-5 if act == torch.float32 else 2e-2
    y_o, fin = O.scan_forward_linear(*ins, st, cs, om, 5, dtype=np.float64)
    assert rel(y.float().cpu().numpy(), y_o) < tol
    assert rel(out[0].cpu().numpy(), fin[0]) < tol
    # float64 autograd reference
    leaf = lambda x: torch.tensor(np.asarray(x, np.float64), requires_grad=True)  # noqa: E731
    ti = [leaf(x) for x in ins]
    ts = (leaf(st[0]), leaf(st[1])) if st is not None else (torch.zeros(B, H, D, D, dtype=torch.float64),
                                                           torch.zeros(B, H, D, D, dtype=torch.float64))
    y_t, (M_t, _) = TR.scan_linear(*ti, ts, cs, om, 5, stop_grad=sg)
    loss = (y_t * torch.as_tensor(dy, dtype=torch.float64)).sum() + (M_t * torch.as_tensor(dM).double()).sum()
    loss.backward()
    names = ["dq", "dk", "dv", "dalpha", "deta", "dtheta", "dgamma"]
    for n, g, ref in zip(names, grads[:7], ti):
        if ref.grad is None:  # gamma is not read without the Omega window
            assert float(g.abs().max()) == 0.0, n
        else:
            assert rel(g.float().cpu().numpy(), ref.grad.numpy()) < tol, n
    if st is not None:
        if sg:
            assert float(grads[7][0].abs().max()) == 0.0 and float(grads[7][1].abs().max()) == 0.0
        else:
            assert rel(grads[7][0].cpu().numpy(), ts[0].grad.numpy()) < tol
            assert rel(grads[7][1].cpu().numpy(), ts[1].grad.numpy()) < tol
