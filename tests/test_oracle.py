"""CPU tests of the oracle: the reference's own known-answer tests, restated,
plus an autograd check of the oracle's hand-written backward."""

import numpy as np
import pytest
import torch

from oracle import atlas_oracle as O
import torch_ref as TR


# --- tests/test_omega.py of the reference ---------------------------------

def test_omega_window_1_is_identity():           # test_omega.py:10-20
    rng = np.random.default_rng(0)
    u = rng.standard_normal((2, 8, 4, 16))
    g = np.ones((2, 8, 4, 1))
    np.testing.assert_allclose(O.omega_aggregate(u, g, 1), g * u, atol=1e-12)


def test_omega_full_window_is_cumsum():          # test_omega.py:23-31
    rng = np.random.default_rng(1)
    u = rng.standard_normal((2, 8, 4, 16))
    np.testing.assert_allclose(O.omega_aggregate(u, np.ones((2, 8, 4, 1)), 8),
                               np.cumsum(u, axis=1), atol=1e-12)


def test_omega_matches_naive():                  # test_omega.py:34-51
    rng = np.random.default_rng(2)
    B, cs, H, D, w = 1, 8, 2, 4, 3
    u = rng.standard_normal((B, cs, H, D))
    g = 1 / (1 + np.exp(-rng.standard_normal((B, cs, H, 1))))
    exp = np.zeros_like(u)
    for t in range(cs):
        for i in range(max(0, t - w + 1), t + 1):
            exp[:, t] += g[:, i] * u[:, i]
    np.testing.assert_allclose(O.omega_aggregate(u, g, w), exp, atol=1e-12)


def test_omega_gamma_zero_masks():               # test_omega.py:54-66  (golden [1,1,2,2])
    u = np.ones((1, 4, 1, 2))
    g = np.array([1.0, 0.0, 1.0, 0.0]).reshape(1, 4, 1, 1)
    np.testing.assert_allclose(O.omega_aggregate(u, g, 4)[0, :, 0, 0], [1, 1, 2, 2])


# --- tests/test_memory_layer.py:17-34 -------------------------------------

def test_linear_scan_basic_recurrence():
    rng = np.random.default_rng(0)
    h0 = rng.standard_normal((2, 2, 3))
    gates = 1 / (1 + np.exp(-rng.standard_normal((2, 4, 2))))
    xs = rng.standard_normal((2, 4, 2, 3))
    h_all, h_fin = O.linear_scan(h0, gates, xs)
    h = h0
    for t in range(4):
        h = gates[:, t, :, None] * h + xs[:, t]
        np.testing.assert_allclose(h_all[:, t], h, atol=1e-12)
    np.testing.assert_allclose(h_fin, h)


# --- tests/test_polar_express.py ------------------------------------------

def test_pe_identity_input():                    # :10-20
    Y = O.polar_express(np.eye(16, dtype=np.float32)[None], 5)
    assert np.std(np.diag(Y[0].T @ Y[0])) < 0.1


def test_pe_output_near_orthogonal():            # :23-34
    X = np.random.default_rng(42).standard_normal((4, 32, 32)).astype(np.float32)
    Y = O.polar_express(X, 5)
    for i in range(4):
        YtY = Y[i].T @ Y[i]
        d = np.diag(YtY)
        assert np.max(np.abs(YtY - np.diag(d))) < 0.5 * np.mean(np.abs(d))


def test_pe_scale_and_shapes():                  # :37-62
    rng = np.random.default_rng(0)
    Y = O.polar_express((rng.standard_normal((2, 16, 16)) * 100).astype(np.float32), 5)
    assert np.all(np.isfinite(Y)) and np.max(np.abs(Y)) < 100
    assert O.polar_express(rng.standard_normal((2, 32, 16)).astype(np.float32)).shape == (2, 32, 16)
    assert O.polar_express(rng.standard_normal((2, 16, 32)).astype(np.float32)).shape == (2, 16, 32)


def test_pe_tall_is_transpose_of_wide():
    """The CUDA kernels store both matrices in one orientation; this identity is why."""
    X = np.random.default_rng(3).standard_normal((3, 64, 16))
    np.testing.assert_allclose(O.polar_express(X), np.swapaxes(O.polar_express(np.swapaxes(X, 1, 2)), 1, 2),
                               rtol=1e-10, atol=1e-12)


def test_pe_batched_consistency():               # :88-95
    X = np.random.default_rng(5).standard_normal((4, 16, 16)).astype(np.float32)
    Yb = O.polar_express(X)
    for i in range(4):
        np.testing.assert_allclose(Yb[i], O.polar_express(X[i:i + 1])[0], atol=1e-5)


def test_pe_vjp_matches_autograd():
    rng = np.random.default_rng(7)
    for shape in [(3, 8, 24), (3, 24, 8)]:
        S = rng.standard_normal(shape)
        G = rng.standard_normal(shape)
        St = torch.tensor(S, requires_grad=True)
        (TR.pe(St, 5) * torch.tensor(G)).sum().backward()
        np.testing.assert_allclose(O.polar_express_vjp(S, G, 5), St.grad.numpy(), rtol=1e-8, atol=1e-10)


# --- full scan: forward vs torch restatement, backward vs autograd --------

def _case(B=1, T=24, H=2, D=4, E=16, seed=0, gamma="random", xavier=True):
    ins = O.make_inputs(B, T, H, D, seed=seed, gamma_mode=gamma)
    st = O.make_xavier_state(B, H, D, E, seed=seed + 1) if xavier else O.lm_initial_state(B, H, D, E)
    # a non-zero momentum carry exercises the S carry paths too
    st = (st[0], st[1], 0.1 * st[0], 0.1 * st[1])
    return ins, st


@pytest.mark.parametrize("T,cs,w,ste,sg", [(24, 8, 3, False, False), (21, 8, 16, False, False),
                                           (16, 8, 1, True, False), (24, 8, 4, False, True)])
def test_scan_forward_backward_vs_autograd(T, cs, w, ste, sg):
    (q, k, v, a, e, t, g), st = _case(T=T)
    y, fin = O.scan_forward(q, k, v, a, e, t, g, st, cs, w, 5, dtype=np.float64)
    tens = [torch.tensor(x.astype(np.float64), requires_grad=True) for x in (q, k, v, a, e, t, g)]
    tst = [torch.tensor(x.astype(np.float64), requires_grad=True) for x in st]
    yt, ft = TR.scan(*tens, tuple(tst), cs, w, 5, ste=ste, stop_grad=sg)
    np.testing.assert_allclose(y, yt.detach().numpy(), rtol=1e-9, atol=1e-9)
    for a_, b_ in zip(fin, ft):
        np.testing.assert_allclose(a_, b_.detach().numpy(), rtol=1e-9, atol=1e-9)
    rng = np.random.default_rng(11)
    dy = rng.standard_normal(y.shape)
    dfin = [rng.standard_normal(x.shape) for x in fin]
    loss = (yt * torch.tensor(dy)).sum() + sum((f * torch.tensor(d)).sum() for f, d in zip(ft, dfin))
    loss.backward()
    grads, dst = O.scan_backward(q, k, v, a, e, t, g, st, dy, dfin, cs, w, 5, pe_ste=ste,
                                 stop_grad_chunks=sg)
    for name, tt in zip(("q", "k", "v", "alpha", "eta", "theta", "gamma"), tens):
        ref = tt.grad.numpy() if tt.grad is not None else np.zeros_like(grads[name])
        if w <= 1 and name == "gamma":
            ref = np.zeros_like(ref)
        np.testing.assert_allclose(grads[name], ref, rtol=1e-7, atol=1e-9, err_msg=name)
    for i, tt in enumerate(tst):
        ref = tt.grad.numpy() if tt.grad is not None else np.zeros_like(dst[i])
        np.testing.assert_allclose(dst[i], ref, rtol=1e-7, atol=1e-9, err_msg=f"state{i}")


def test_padding_zeroes_momentum_carry():
    """memory_layer.py:649-660: pad tokens have theta = 0, so S in the final carry is 0."""
    (q, k, v, a, e, t, g), st = _case(T=13)
    _, fin = O.scan_forward(q, k, v, a, e, t, g, st, 8, 4, 5)
    assert np.all(fin[2] == 0) and np.all(fin[3] == 0)


def test_state_resume():
    """scan(T1+T2) == scan(T2, state=scan(T1)) when T1 is a chunk multiple."""
    (q, k, v, a, e, t, g), st = _case(T=32)
    y, fin = O.scan_forward(q, k, v, a, e, t, g, st, 8, 4, 5, dtype=np.float64)
    sl1, sl2 = slice(0, 16), slice(16, 32)
    y1, s1 = O.scan_forward(q[:, sl1], k[:, sl1], v[:, sl1], a[:, sl1], e[:, sl1], t[:, sl1], g[:, sl1],
                            st, 8, 4, 5, dtype=np.float64)
    y2, s2 = O.scan_forward(q[:, sl2], k[:, sl2], v[:, sl2], a[:, sl2], e[:, sl2], t[:, sl2], g[:, sl2],
                            s1, 8, 4, 5, dtype=np.float64)
    np.testing.assert_allclose(np.concatenate([y1, y2], 1), y, rtol=1e-12, atol=1e-12)


def test_oracle_matches_golden_config0():
    """The committed config-0 vectors (tests/golden/make_golden.py) still match."""
    import os
    gold = np.load(os.path.join(os.path.dirname(__file__), "golden", "config0.npz"))
    q, k, v, a, e, t, g = O.make_inputs(2, 512, 4, 32, seed=0, gamma_mode="ones")
    y, fin = O.scan_forward(q, k, v, a, e, t, g, O.lm_initial_state(2, 4, 32, 128), 64, 8, 5,
                            dtype=np.float64)
    rel = np.linalg.norm(y - gold["lm_y"]) / np.linalg.norm(gold["lm_y"])
    assert rel < 1e-6
    for n, x in zip(("W1", "W2", "S1", "S2"), fin):
        assert np.linalg.norm(x - gold[f"lm_{n}"]) <= 1e-6 * np.linalg.norm(gold[f"lm_{n}"])


def test_gamma_none_means_ones():
    """A missing gamma gate is all ones, as a NULL gamma at the C ABI."""
    ins = O.make_inputs(1, 70, 2, 16, seed=5)
    st = O.lm_initial_state(1, 2, 16, 64)
    y1, s1 = O.scan_forward(*ins[:6], None, st, 32, 4, 2)
    y2, s2 = O.scan_forward(*ins[:6], np.ones_like(ins[5]), st, 32, 4, 2)
    assert np.array_equal(y1, y2) and all(np.array_equal(a, b) for a, b in zip(s1, s2))


def test_layer_prologue_oracle_matches_torch_restatement():
    """oracle.layer_prologue (numpy) against tests/layer_ref.py (torch conv1d), float64."""
    import torch
    import layer_ref as LR
    B, T, H, D, K = 2, 9, 2, 16, 4
    rng = np.random.default_rng(0)
    for P, hg, hr in ((2, True, True), (0, False, False), (3, True, False)):
        G = 3 + hg + hr
        proj = rng.standard_normal((B * T, 3 * H * D + G * H))
        cw, cb, poly, gb = LR.make_params(H, D, K, P, G - hr)
        a = O.layer_prologue(proj, B, T, H, D, cw.astype(np.float64), cb.astype(np.float64),
                             None if poly is None else poly.astype(np.float64), gb.astype(np.float64), hg, hr, 0.1)
        t = lambda x: None if x is None else torch.as_tensor(x, dtype=torch.float64)  # noqa: E731
        b = LR.prologue(t(proj), B, T, H, D, t(cw), t(cb), t(poly), t(gb), hg, hr, 0.1)
        for x, y in zip(a[:3], b[:3]):
            np.testing.assert_allclose(x, y.numpy(), rtol=1e-12, atol=1e-12)
        for x, y in zip(a[3], b[3]):
            assert (x is None) == (y is None)
            if x is not None:
                np.testing.assert_allclose(x, y.numpy(), rtol=1e-12, atol=1e-14)


def test_linear_torch_restatement_matches_oracle_forward():
    """tests/torch_ref.scan_linear (the autograd checker of the linear backward) equals
    the oracle's linear forward in float64."""
    import torch
    import torch_ref as TR
    B, T, H, D = 1, 40, 2, 8
    ins = O.make_inputs(B, T, H, D, seed=4, gamma_mode="random")
    rng = np.random.default_rng(1)
    st = (0.1 * rng.standard_normal((B, H, D, D)), 0.01 * rng.standard_normal((B, H, D, D)))
    y_o, fin = O.scan_forward_linear(*ins, st, 16, 4, 5, dtype=np.float64)
    t = [torch.as_tensor(np.asarray(x, np.float64)) for x in ins]
    y_t, fin_t = TR.scan_linear(*t, tuple(torch.as_tensor(x) for x in st), 16, 4, 5)
    np.testing.assert_allclose(y_t.numpy(), y_o, rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(fin_t[0].numpy(), fin[0], rtol=1e-10, atol=1e-12)
