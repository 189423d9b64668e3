"""Independent torch (CPU, float64) restatement of the reference scan, used only
to check the oracle's hand-written backward by autograd.

Follows atlas_jax/memory_layer.py:43-71 (Polar Express), 225-253 (GELU', Omega),
256-299 (linear scan), 496-597 (deep chunk body) and 649-718 (driver, padding).
"""

import math

import torch

COEFFS = [
    (8.156554524902461, -22.48329292557795, 15.878769915207462),
    (4.042929935166739, -2.808917465908714, 0.5000178451051316),
    (3.8916678022926607, -2.772484153217685, 0.5060648178503393),
    (3.285753657755655, -2.3681294933425376, 0.46449024233003106),
    (2.3465413258596377, -1.7097828382687081, 0.42323551169305323),
]


def gelu_tanh(x):
    return 0.5 * x * (1.0 + torch.tanh(math.sqrt(2.0 / math.pi) * (x + 0.044715 * x ** 3)))


def gelu_prime(x):
    return 0.5 * (1.0 + torch.erf(x * 0.7071067811865476)) + x * torch.exp(-0.5 * x * x) * 0.3989422804014327


def pe(X, steps, ste=False):
    n = torch.sqrt((X * X).sum(dim=(-2, -1), keepdim=True) + 1e-12)
    Y = X / (n * 1.01 + 1e-6)
    tall = Y.shape[-2] > Y.shape[-1]
    for a, b, c in COEFFS[:steps]:
        if tall:
            A = Y.transpose(-2, -1) @ Y
            Bm = b * A + c * (A @ A)
            Y = a * Y + Y @ Bm
        else:
            A = Y @ Y.transpose(-2, -1)
            Bm = b * A + c * (A @ A)
            Y = a * Y + Bm @ Y
    if ste:
        return X + (Y - X).detach()
    return Y


def omega(u, g, w):
    cs = u.shape[1]
    cum = torch.cumsum(g * u, dim=1)
    if w >= cs:
        return cum
    sh = torch.cat([torch.zeros_like(cum[:, :w]), cum[:, :-w]], dim=1)
    return cum - sh


def lscan(h, gates, xs):
    outs = []
    g = gates.reshape(gates.shape + (1,) * (xs.ndim - gates.ndim))
    for t in range(xs.shape[1]):
        h = g[:, t] * h + xs[:, t]
        outs.append(h)
    return torch.stack(outs, 1), h


def chunk(state, q, k, v, a, e, t, g, w, ns, ste):
    W1, W2, S1, S2 = state
    D = k.shape[-1]
    h = torch.einsum('bhed,bchd->bche', W2, k)
    act = gelu_tanh(h)
    err = k + torch.einsum('bhde,bche->bchd', W1, act) - v
    u1 = (2.0 / D) * torch.einsum('bchd,bche->bchde', err, act)
    chain = torch.einsum('bhde,bchd->bche', W1, err) * gelu_prime(h)
    u2 = (2.0 / D) * torch.einsum('bche,bchd->bched', chain, k)
    if w > 1:
        u1 = omega(u1, g[..., None, None], w)
        u2 = omega(u2, g[..., None, None], w)
    m1 = -(e[..., None, None] * u1)
    m2 = -(e[..., None, None] * u2)
    S1a, S1 = lscan(S1, t, m1)
    S2a, S2 = lscan(S2, t, m2)
    W1a, W1 = lscan(W1, a, pe(S1a, ns, ste))
    W2a, W2 = lscan(W2, a, pe(S2a, ns, ste))
    hq = torch.einsum('bched,bchd->bche', W2a, q)
    y = q + torch.einsum('bchde,bche->bchd', W1a, gelu_tanh(hq))
    return y, (W1, W2, S1, S2)


def scan(q, k, v, a, e, t, g, state, cs, w, ns, ste=False, stop_grad=False):
    T = q.shape[1]
    pad = (-T) % cs

    def p(x, val):
        if pad == 0:
            return x
        shape = list(x.shape)
        shape[1] = pad
        return torch.cat([x, torch.full(shape, val, dtype=x.dtype, device=x.device)], 1)
    q, k, v = p(q, 0.0), p(k, 0.0), p(v, 0.0)
    a, e, t, g = p(a, 1.0), p(e, 0.0), p(t, 0.0), p(g, 0.0)
    ys = []
    st = state
    for c in range(q.shape[1] // cs):
        sl = slice(c * cs, (c + 1) * cs)
        if stop_grad:
            st = tuple(x.detach() for x in st)
        y, st = chunk(st, q[:, sl], k[:, sl], v[:, sl], a[:, sl], e[:, sl], t[:, sl], g[:, sl], w, ns, ste)
        ys.append(y)
    return torch.cat(ys, 1)[:, :T], st


def chunk_linear(state, q, k, v, a, e, t, g, w, ns, ste):
    """Linear-memory chunk body, memory_layer.py:468-494."""
    M, S = state
    D = k.shape[-1]
    err = torch.einsum('bhvk,bchk->bchv', M, k) - v
    u = (2.0 / D) * torch.einsum('bchv,bchk->bchvk', err, k)
    if w > 1:
        u = omega(u, g[..., None, None], w)
    Sa, S = lscan(S, t, -(e[..., None, None] * u))
    Ma, M = lscan(M, a, pe(Sa, ns, ste))
    return torch.einsum('bchvk,bchk->bchv', Ma, q), (M, S)


def scan_linear(q, k, v, a, e, t, g, state, cs, w, ns, ste=False, stop_grad=False):
    """Driver 649-718 over the linear chunk body (state (M, S))."""
    T = q.shape[1]
    pad = (-T) % cs

    def p(x, val):
        if pad == 0:
            return x
        shape = list(x.shape)
        shape[1] = pad
        return torch.cat([x, torch.full(shape, val, dtype=x.dtype, device=x.device)], 1)
    q, k, v = p(q, 0.0), p(k, 0.0), p(v, 0.0)
    a, e, t, g = p(a, 1.0), p(e, 0.0), p(t, 0.0), p(g, 0.0)
    ys, st = [], state
    for c in range(q.shape[1] // cs):
        sl = slice(c * cs, (c + 1) * cs)
        if stop_grad:
            st = tuple(x.detach() for x in st)
        y, st = chunk_linear(st, q[:, sl], k[:, sl], v[:, sl], a[:, sl], e[:, sl], t[:, sl], g[:, sl], w, ns, ste)
        ys.append(y)
    return torch.cat(ys, 1)[:, :T], st
