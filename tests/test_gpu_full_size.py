"""Full-size launch of the tcgen05 scan at the 170M configuration (B=8, T=8192, H=12,
D=64, E=256, chunk 64, Omega 16, 5 Newton-Schulz steps, bf16 activations), checked
through properties that do not need the oracle to run at that size:

* causality: the first P tokens of every chain depend only on those tokens, so the
  full launch's outputs there must equal the float64 oracle run on the P-token prefix
  alone (a few chains are checked);
* the same holds for the backward when dy is zero from token P on: the prefix's
  input gradients and the initial-state gradient match the oracle's prefix VJP;
* every output of the full launch is finite.

The launch covers every cluster of the persistent grid, chains migrating between
clusters, and the full-size workspace and saved-carry buffers.  Tolerance 2e-2
relative (the bf16-activation bound), as in the other tensor-path tests.
"""
import numpy as np
import pytest
import torch

from oracle import atlas_oracle as O
from gpu_util import rel, to_np

pytestmark = pytest.mark.gpu
TOL = 2e-2
B, T, H, D, E, CS, OM, NS = 8, 8192, 12, 64, 256, 64, 16, 5
P = 128  # prefix checked against the oracle
CHAINS = [(0, 0), (3, 7), (7, 11)]


def test_full_size_prefix_parity_and_finite():
    from atlas_b200 import ScanConfig, ATLAS_PREC_TENSOR, scan_forward, scan_backward, device_status
    g = torch.Generator(device="cuda").manual_seed(123)

    def unit(x):
        return x / x.norm(dim=-1, keepdim=True)

    q, k, v = [unit(torch.randn(B, T, H, D, device="cuda", generator=g)).to(torch.bfloat16) for _ in range(3)]

    def gate(mu):
        return torch.sigmoid(mu + 0.5 * torch.randn(B, T, H, device="cuda", generator=g))

    al, et, th, ga = gate(3.0), gate(-3.0), gate(1.0), gate(0.0)
    cfg = ScanConfig(chunk=CS, omega=OM, ns_steps=NS, precision=ATLAS_PREC_TENSOR)
    y, st, saved = scan_forward(q, k, v, al, et, th, ga, None, cfg)
    dy = torch.zeros_like(y)
    dy[:, :P] = torch.randn(B, P, H, D, device="cuda", generator=g).to(torch.bfloat16)
    res = scan_backward(q, k, v, al, et, th, ga, saved, dy, None, cfg, E)
    torch.cuda.synchronize()
    device_status()

    for name, x in [("y", y), ("dq", res[0]), ("dk", res[1]), ("dv", res[2])] + \
            [(n, res[3 + i]) for i, n in enumerate(("dalpha", "deta", "dtheta", "dgamma"))] + \
            [(f"state{i}", s) for i, s in enumerate(st)] + [(f"dstate{i}", s) for i, s in enumerate(res[7])]:
        assert bool(torch.isfinite(x).all()), name

    st0 = O.lm_initial_state(1, 1, D, E)
    for b, h in CHAINS:
        sl = lambda x: to_np(x[b:b + 1, :P, h:h + 1]).astype(np.float64)  # noqa: E731
        ins = [sl(x) for x in (q, k, v, al, et, th, ga)]
        y_o, _ = O.scan_forward(*ins, st0, CS, OM, NS, dtype=np.float64)
        grads, dst = O.scan_backward(*ins, st0, sl(dy), None, CS, OM, NS)
        errs = {"y": rel(sl(y), y_o)}
        for i, n in enumerate(("q", "k", "v", "alpha", "eta", "theta", "gamma")):
            errs["d" + n] = rel(sl(res[i]), grads[n])
        for i, n in enumerate(("dW1", "dW2", "dS1", "dS2")):
            if np.abs(dst[i]).max() > 0:
                errs[n] = rel(to_np(res[7][i][b:b + 1, h:h + 1]), dst[i])
        print((b, h), {k_: f"{v_:.2e}" for k_, v_ in errs.items()})
        assert max(errs.values()) < TOL, ((b, h), errs)
