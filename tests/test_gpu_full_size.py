"""Full-size launch of the tcgen05 scan at the 170M configuration (B=8, T=8192, H=12,
D=64, E=256, chunk 64, Omega 16, 5 Newton-Schulz steps, bf16 activations), checked
chunk by chunk against the float64 oracle:

* forward: for 16 (chain, chunk) pairs spread over all 96 chains (chunk 0 and the
  last chunk 127 among them) the oracle runs that chunk alone from the carry the
  kernel stored in ``saved`` for it; the chunk's 64 outputs y must match, and so must
  the carry out (``saved`` of the next chunk, or the final state after chunk 127);
* one whole chain runs through the oracle from the initial state, window by window,
  for as long as the reference's own float32 arithmetic stays near float64 (the scan
  is chaotic: rounding differences grow about 5x per 256 tokens);
* backward: dy is non-zero in a single chunk c_q of each checked chain, so the
  cotangent of the carry leaving c_q is zero and the input gradients of c_q's tokens
  are the oracle's VJP of that one chunk from its saved carry (memory_layer.py:664-711);
* every output of the full launch is finite.

The launch covers every cluster of the persistent grid, chains migrating between
clusters late in the wavefront, and the full-size workspace and saved buffers.
Tolerance 2e-2 relative (the bf16-activation bound); each checked chunk's errors are
printed.
"""
import numpy as np
import pytest
import torch

from oracle import atlas_oracle as O
from gpu_util import rel, to_np

pytestmark = pytest.mark.gpu
TOL = 2e-2
B, T, H, D, E, CS, OM, NS = 8, 8192, 12, 64, 256, 64, 16, 5
NCH = T // CS
DE = D * E
_rng = np.random.default_rng(2024)
_chains = _rng.choice(B * H, size=16, replace=False)
_chunks = _rng.integers(1, NCH - 1, size=16)
_chunks[0], _chunks[1] = 0, NCH - 1
PAIRS = [(int(q), int(c)) for q, c in zip(_chains, _chunks)]
FULL_CHAIN = int(_chains[2])


def _carry(saved, q, c):
    """Carry entering chunk c of chain q, from the kernel's `saved` buffer
    ([chain][chunk][matrix][W, S][E x D], W1 / S1 stored transposed), oracle layout."""
    sl = saved.view(torch.float32).view(B * H, NCH, 2, 2, E, D)[q, c].double().cpu().numpy()
    W1, S1 = sl[0, 0].T[None, None], sl[0, 1].T[None, None]
    W2, S2 = sl[1, 0][None, None], sl[1, 1][None, None]
    return W1, W2, S1, S2


def test_full_size_chunkwise_parity_and_finite():
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
    # dy: random everywhere for unchecked chains, one chunk only for the checked ones
    dy = (0.01 * torch.randn(B, T, H, D, device="cuda", generator=g)).to(torch.bfloat16)
    for qq, c in PAIRS:
        b, h = divmod(qq, H)
        keep = dy[b, c * CS:(c + 1) * CS, h].clone()
        dy[b, :, h] = 0
        dy[b, c * CS:(c + 1) * CS, h] = keep
    res = scan_backward(q, k, v, al, et, th, ga, saved, dy, None, cfg, E)
    torch.cuda.synchronize()
    device_status()

    for name, x in [("y", y), ("dq", res[0]), ("dk", res[1]), ("dv", res[2])] + \
            [(n, res[3 + i]) for i, n in enumerate(("dalpha", "deta", "dtheta", "dgamma"))] + \
            [(f"state{i}", s) for i, s in enumerate(st)] + [(f"dstate{i}", s) for i, s in enumerate(res[7])]:
        assert bool(torch.isfinite(x).all()), name

    worst = 0.0
    for qq, c in PAIRS:
        b, h = divmod(qq, H)
        tok = slice(c * CS, (c + 1) * CS)
        sl = lambda x: to_np(x[b:b + 1, tok, h:h + 1]).astype(np.float64)  # noqa: E731
        ins = [sl(x) for x in (q, k, v, al, et, th, ga)]
        carry = _carry(saved, qq, c)
        y_o, nxt = O.chunk_forward(carry, *ins, OM, NS)
        errs = {"y": rel(sl(y), y_o)}
        if c + 1 < NCH:
            after = _carry(saved, qq, c + 1)
        else:
            after = tuple(to_np(s_[b:b + 1, h:h + 1]).astype(np.float64) for s_ in st)
        for i, n in enumerate(("W1", "W2", "S1", "S2")):
            errs["carry_" + n] = rel(after[i], nxt[i])
        zeros = tuple(np.zeros_like(x) for x in carry)
        gr, _ = O.chunk_backward(carry, *ins, sl(dy), zeros, OM, NS)
        for i, n in enumerate(("q", "k", "v", "alpha", "eta", "theta", "gamma")):
            errs["d" + n] = rel(sl(res[i]), gr[n])
        print((qq, c), {k_: f"{v_:.2e}" for k_, v_ in errs.items()})
        worst = max(worst, max(errs.values()))
        assert max(errs.values()) < TOL, ((qq, c), errs)
    print("worst chunk error", worst)

    # one whole chain from the LM initial state.  The scan is chaotic over long
    # horizons: rounding differences grow about 5x per 256 tokens (the reference's
    # own float32 forward leaves its float64 one by 100 % after ~1500 tokens), so a
    # whole-sequence comparison checks the kernel window by window against the
    # envelope of that growth: in every 256-token window up to the point where the
    # float32 oracle has drifted 10 % from the float64 one, the kernel must be within
    # max(2e-2, 4 x the float32 oracle's drift) of the float64 oracle.
    b, h = divmod(FULL_CHAIN, H)
    n_win = 8
    ins = [to_np(x[b:b + 1, :n_win * 256, h:h + 1]).astype(np.float64) for x in (q, k, v, al, et, th, ga)]
    st0 = O.lm_initial_state(1, 1, D, E, np.float64)
    y64, _ = O.scan_forward(*ins, st0, CS, OM, NS, dtype=np.float64)
    y32, _ = O.scan_forward(*ins, st0, CS, OM, NS, dtype=np.float32)
    yk = to_np(y[b:b + 1, :n_win * 256, h:h + 1])
    checked = 0
    for wdw in range(n_win):
        sw = slice(256 * wdw, 256 * (wdw + 1))
        drift = rel(y32[:, sw], y64[:, sw])
        if drift > 0.1:
            break
        err = rel(yk[:, sw], y64[:, sw])
        print(f"full chain {FULL_CHAIN} window {wdw}: kernel {err:.2e}, float32 oracle drift {drift:.2e}")
        assert err <= max(TOL, 4 * drift), (wdw, err, drift)
        checked += 1
    assert checked >= 3
