"""CPU oracle for the Atlas chunked deep-memory scan (TEST INFRASTRUCTURE ONLY).

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s ``cpu_baseline`` / ``--impl
reference`` leg may import it.  The shipped path is the CUDA library behind
``include/atlas_scan.h`` and fails loudly when that library is missing.

It restates, in numpy, the reference's pure-JAX (non-fused) scan of
rkstgr/atlas-jax:

* Polar Express            -- atlas_jax/memory_layer.py:34-71 (coefficients 34-40,
                              Frobenius pre-normalisation 55-56, tall/wide 60-69);
                              identical math to atlas_jax/kernels/triton_pe.py:26-69.
* STE variant              -- memory_layer.py:74-76
* exact GELU derivative    -- memory_layer.py:225-230
* Omega window aggregation -- memory_layer.py:233-253 (cumsum minus shifted cumsum)
* linear recurrence        -- memory_layer.py:256-299
* deep chunk body          -- memory_layer.py:496-597 (D != E branch 577-590)
* linear-memory chunk body -- memory_layer.py:468-494
* scan driver / padding    -- memory_layer.py:649-718
* LM-path initial state    -- atlas_jax/model.py:251-264

The backward pass is a hand-written vector-Jacobian product of the same
restatement (the reference obtains it from JAX autodiff with per-chunk
``jax.checkpoint``, memory_layer.py:675).  It is cross-checked in the tests
against torch float64 autograd of an independent restatement and against
finite differences.

Parity pinning: the reference ships no golden vectors for the full scan and
JAX is not installed in this image, so full-scan parity is pinned only through
the reference's own sub-step known-answer tests (tests/test_omega.py,
tests/test_memory_layer.py:17-34, tests/test_polar_express.py) which
``tests/test_oracle.py`` re-runs against this module.

Arrays: q, k, v are (B, T, H, D); gates alpha, eta, theta, gamma are (B, T, H);
state W1, S1 are (B, H, D, E) and W2, S2 are (B, H, E, D) -- the reference's
naming, in which W2 is the first MLP layer: M(x) = x + W1 gelu(W2 x).
"""

import math

import numpy as np

# memory_layer.py:34-40
POLAR_EXPRESS_COEFFS = [
    (8.156554524902461, -22.48329292557795, 15.878769915207462),
    (4.042929935166739, -2.808917465908714, 0.5000178451051316),
    (3.8916678022926607, -2.772484153217685, 0.5060648178503393),
    (3.285753657755655, -2.3681294933425376, 0.46449024233003106),
    (2.3465413258596377, -1.7097828382687081, 0.42323551169305323),
]

_SQRT_2_OVER_PI = math.sqrt(2.0 / math.pi)


def _erf(x):
    # numpy has no erf; math.erf vectorised keeps double precision.
    return np.vectorize(math.erf, otypes=[np.float64])(x)


try:  # scipy is present in the image; fall back to math.erf otherwise
    from scipy.special import erf as _scipy_erf

    def _erf(x):  # noqa: F811
        return _scipy_erf(np.asarray(x, dtype=np.float64))
except Exception:  # pragma: no cover
    pass


# ---------------------------------------------------------------------------
# elementwise functions
# ---------------------------------------------------------------------------

def gelu_tanh(x):
    """jax.nn.gelu default (approximate=True), used at memory_layer.py:506, 594."""
    u = _SQRT_2_OVER_PI * (x + 0.044715 * x ** 3)
    return 0.5 * x * (1.0 + np.tanh(u))


def gelu_tanh_grad(x):
    """d/dx of gelu_tanh (what JAX autodiff differentiates for 506 / 594)."""
    u = _SQRT_2_OVER_PI * (x + 0.044715 * x ** 3)
    t = np.tanh(u)
    du = _SQRT_2_OVER_PI * (1.0 + 3.0 * 0.044715 * x * x)
    return 0.5 * (1.0 + t) + 0.5 * x * (1.0 - t * t) * du


def gelu_erf_prime(x):
    """Exact derivative of x*Phi(x): memory_layer.py:225-230."""
    xd = np.asarray(x, dtype=np.float64)
    cdf = 0.5 * (1.0 + _erf(xd * 0.7071067811865476))
    pdf = np.exp(-0.5 * xd * xd) * 0.3989422804014327
    return (cdf + xd * pdf).astype(np.result_type(x, np.float32))


def gelu_erf_second(x):
    """d/dx of gelu_erf_prime: (2 - x^2) * phi(x)  (needed by the backward)."""
    xd = np.asarray(x, dtype=np.float64)
    pdf = np.exp(-0.5 * xd * xd) * 0.3989422804014327
    return ((2.0 - xd * xd) * pdf).astype(np.result_type(x, np.float32))


# ---------------------------------------------------------------------------
# Polar Express
# ---------------------------------------------------------------------------

def _pe_norm_scale(S):
    """memory_layer.py:55-56: X = S / (||S||_F * 1.01 + 1e-6), ||S|| = sqrt(sum S^2 + 1e-12)."""
    n = np.sqrt(np.sum(S * S, axis=(-2, -1), keepdims=True) + 1e-12)
    kappa = n * 1.01 + 1e-6
    return n, kappa


def polar_express(X, steps=5, keep=False):
    """Batched Polar Express, memory_layer.py:43-71.

    ``X`` is (..., d1, d2) and is computed in its own float dtype (the
    reference casts to float32 first; pass float64 for the gradient checks).
    With ``keep`` the per-step intermediates are returned for the VJP.
    """
    dt = X.dtype if X.dtype in (np.float32, np.float64) else np.float32
    X = X.astype(dt)
    n, kappa = _pe_norm_scale(X)
    X = X / kappa
    d1, d2 = X.shape[-2], X.shape[-1]
    tall = d1 > d2
    hist = []
    for a, b, c in POLAR_EXPRESS_COEFFS[:steps]:
        a, b, c = dt.type(a), dt.type(b), dt.type(c)
        if tall:
            A = np.swapaxes(X, -2, -1) @ X          # memory_layer.py:62
        else:
            A = X @ np.swapaxes(X, -2, -1)          # memory_layer.py:67
        Bm = b * A + c * (A @ A)                    # 63 / 68
        hist.append((X, A, Bm))
        X = a * X + (X @ Bm if tall else Bm @ X)    # 64 / 69
    if keep:
        return X, (n, kappa, tall, hist)
    return X


def polar_express_vjp(S, dO, steps=5):
    """VJP of ``polar_express`` (JAX autodiff of memory_layer.py:43-71)."""
    dt = S.dtype
    _, (n, kappa, tall, hist) = polar_express(S, steps, keep=True)
    G = dO.astype(dt)
    T = lambda M: np.swapaxes(M, -2, -1)  # noqa: E731
    for (a, b, c), (X, A, Bm) in reversed(list(zip(POLAR_EXPRESS_COEFFS[:steps], hist))):
        a, b, c = dt.type(a), dt.type(b), dt.type(c)
        if tall:
            # X' = a X + X B,  A = X^T X
            dX = a * G + G @ T(Bm)
            dB = T(X) @ G
        else:
            # X' = a X + B X,  A = X X^T
            dX = a * G + T(Bm) @ G
            dB = G @ T(X)
        dA = b * dB + c * (dB @ T(A) + T(A) @ dB)
        if tall:
            dX = dX + X @ (dA + T(dA))
        else:
            dX = dX + (dA + T(dA)) @ X
        G = dX
    # X0 = S / kappa, kappa = 1.01 * sqrt(sum S^2 + 1e-12) + 1e-6
    dot = np.sum(G * S, axis=(-2, -1), keepdims=True)
    dS = G / kappa - (dot / (kappa * kappa)) * 1.01 * S / n
    return dS


def polar_express_ste(X, steps=5):
    """memory_layer.py:74-76 -- forward equals ``polar_express``; gradient is identity."""
    return polar_express(X, steps)


# ---------------------------------------------------------------------------
# scan primitives
# ---------------------------------------------------------------------------

def omega_aggregate(u, gamma, omega_window):
    """memory_layer.py:233-253.  u: (B, cs, H, ...), gamma broadcastable to u."""
    cs = u.shape[1]
    cum = np.cumsum(gamma * u, axis=1)
    if omega_window >= cs:
        return cum
    shifted = np.concatenate([np.zeros_like(cum[:, :omega_window]),
                              cum[:, :-omega_window]], axis=1)
    return cum - shifted


def linear_scan(h_init, gates, inputs):
    """memory_layer.py:256-299 (h_t = g_t h_{t-1} + x_t), as the sequential loop
    of tests/test_memory_layer.py:17-34.  gates: (B, T, H); inputs (B, T, H, ...)."""
    extra = inputs.ndim - gates.ndim
    g = gates.reshape(gates.shape + (1,) * extra)
    h = h_init
    out = np.empty_like(inputs)
    for t in range(inputs.shape[1]):
        h = g[:, t] * h + inputs[:, t]
        out[:, t] = h
    return out, h


def _ein(spec, *ops):
    return np.einsum(spec, *ops, optimize=True)


# ---------------------------------------------------------------------------
# one chunk, forward (memory_layer.py:496-597)
# ---------------------------------------------------------------------------

def chunk_forward(state, q, k, v, a, e, t, g, omega, ns_steps, keep=False):
    """Deep-memory chunk body.  q,k,v: (B,cs,H,D); a,e,t,g: (B,cs,H).

    Returns (y, new_state[, intermediates]).  All math in the dtype of the
    state (float32 like the reference's f32 path, or float64 for checks)."""
    W1, W2, S1, S2 = state
    dt = W1.dtype
    D = k.shape[-1]
    s = dt.type(2.0 / D)
    # mem_fwd 504-508
    h = _ein('bhed,bchd->bche', W2, k)
    act = gelu_tanh(h)
    err = k + _ein('bhde,bche->bchd', W1, act) - v
    # mem_grad 510-520
    u1 = s * _ein('bchd,bche->bchde', err, act)
    gp = gelu_erf_prime(h).astype(dt)
    w1t_err = _ein('bhde,bchd->bche', W1, err)
    chain = w1t_err * gp
    u2 = s * _ein('bche,bchd->bched', chain, k)
    # omega 522-527
    if omega > 1:
        G1 = omega_aggregate(u1, g[..., None, None], omega)
        G2 = omega_aggregate(u2, g[..., None, None], omega)
    else:
        G1, G2 = u1, u2
    # momentum 529-533
    m1 = -(e[..., None, None] * G1)
    m2 = -(e[..., None, None] * G2)
    # _fused_scan 578-590
    S1_all, S1n = linear_scan(S1, t, m1)
    S2_all, S2n = linear_scan(S2, t, m2)
    O1 = polar_express(S1_all, ns_steps)
    O2 = polar_express(S2_all, ns_steps)
    W1_all, W1n = linear_scan(W1, a, O1)
    W2_all, W2n = linear_scan(W2, a, O2)
    # mem_output 592-595
    hq = _ein('bched,bchd->bche', W2_all, q)
    gq = gelu_tanh(hq)
    y = q + _ein('bchde,bche->bchd', W1_all, gq)
    new_state = (W1n, W2n, S1n, S2n)
    if not keep:
        return y, new_state
    inter = dict(h=h, act=act, err=err, u1=u1, u2=u2, gp=gp, w1t_err=w1t_err,
                 chain=chain, G1=G1, G2=G2, S1_all=S1_all, S2_all=S2_all,
                 O1=O1, O2=O2, W1_all=W1_all, W2_all=W2_all, hq=hq, gq=gq)
    return y, new_state, inter


def chunk_forward_linear(state, q, k, v, a, e, t, g, omega, ns_steps):
    """Linear-memory chunk body, memory_layer.py:468-494: pred = M k, u = (2/D) err k^T,
    Omega window, S scan, square Polar Express, M scan, y = M_t q (no residual)."""
    M, S = state
    dt = M.dtype
    D = k.shape[-1]
    pred = _ein('bhvk,bchk->bchv', M, k)
    err = pred - v
    u = dt.type(2.0 / D) * _ein('bchv,bchk->bchvk', err, k)
    if omega > 1:
        u = omega_aggregate(u, g[..., None, None], omega)
    mom = -(e[..., None, None] * u)
    S_all, S_n = linear_scan(S, t, mom)
    O = polar_express(S_all, ns_steps)
    M_all, M_n = linear_scan(M, a, O)
    y = _ein('bchvk,bchk->bchv', M_all, q)
    return y, (M_n, S_n)


def scan_forward_linear(q, k, v, alpha, eta, theta, gamma, state=None, chunk=64, omega=16, ns_steps=5,
                        dtype=np.float32):
    """Whole-sequence linear-memory forward (driver memory_layer.py:649-718 with the
    linear chunk body); state None = zeros (memory_layer.py:138-140, 644-646)."""
    T, q, k, v, alpha, eta, theta, gamma = _prepare(q, k, v, alpha, eta, theta, gamma, chunk, dtype)
    B, _, H, D = q.shape
    if state is None:
        state = (np.zeros((B, H, D, D), dtype), np.zeros((B, H, D, D), dtype))
    st = tuple(np.asarray(x).astype(dtype) for x in state)
    ys = []
    for c in range(q.shape[1] // chunk):
        sl = slice(c * chunk, (c + 1) * chunk)
        y_c, st = chunk_forward_linear(st, q[:, sl], k[:, sl], v[:, sl], alpha[:, sl], eta[:, sl],
                                       theta[:, sl], gamma[:, sl], omega, ns_steps)
        ys.append(y_c)
    return np.concatenate(ys, axis=1)[:, :T], st


def _rev_linear_scan(gates, dh_all, dh_final, h_prev_all):
    """VJP of ``linear_scan``: returns (d_inputs, d_gates, d_h_init).

    h_prev_all[:, t] is h_{t-1} (h_init at t=0)."""
    extra = dh_all.ndim - gates.ndim
    g = gates.reshape(gates.shape + (1,) * extra)
    acc = dh_final.copy()
    dx = np.empty_like(dh_all)
    dg = np.empty(gates.shape, dtype=dh_all.dtype)
    for t in range(dh_all.shape[1] - 1, -1, -1):
        acc = acc + dh_all[:, t]
        dx[:, t] = acc
        dg[:, t] = np.sum(acc * h_prev_all[:, t], axis=tuple(range(2, acc.ndim)))
        acc = g[:, t] * acc
    return dx, dg, acc


def _shift_prev(h_init, h_all):
    return np.concatenate([h_init[:, None], h_all[:, :-1]], axis=1)


def chunk_backward(state, q, k, v, a, e, t, g, dy, dstate, omega, ns_steps,
                   pe_ste=False):
    """VJP of ``chunk_forward`` with respect to every input and the incoming carry."""
    W1, W2, S1, S2 = state
    dW1n, dW2n, dS1n, dS2n = dstate
    dt = W1.dtype
    D = k.shape[-1]
    s = dt.type(2.0 / D)
    _, _, I = chunk_forward(state, q, k, v, a, e, t, g, omega, ns_steps, keep=True)

    # mem_output: y = q + W1_t gelu(W2_t q)
    dW1_all = _ein('bchd,bche->bchde', dy, I['gq'])
    dgq = _ein('bchde,bchd->bche', I['W1_all'], dy)
    dhq = dgq * gelu_tanh_grad(I['hq'])
    dW2_all = _ein('bche,bchd->bched', dhq, q)
    dq = dy + _ein('bched,bche->bchd', I['W2_all'], dhq)

    # memory scans W_t = a_t W_{t-1} + O_t
    dO1, da1, dW1_in = _rev_linear_scan(a, dW1_all, dW1n, _shift_prev(W1, I['W1_all']))
    dO2, da2, dW2_in = _rev_linear_scan(a, dW2_all, dW2n, _shift_prev(W2, I['W2_all']))
    da = da1 + da2

    # Polar Express
    if pe_ste:
        dSa1, dSa2 = dO1, dO2
    else:
        dSa1 = polar_express_vjp(I['S1_all'], dO1, ns_steps)
        dSa2 = polar_express_vjp(I['S2_all'], dO2, ns_steps)

    # momentum scans S_t = t_t S_{t-1} + m_t
    dm1, dt1, dS1_in = _rev_linear_scan(t, dSa1, dS1n, _shift_prev(S1, I['S1_all']))
    dm2, dt2, dS2_in = _rev_linear_scan(t, dSa2, dS2n, _shift_prev(S2, I['S2_all']))
    dth = dt1 + dt2

    # m = -e * G
    de = -(np.sum(dm1 * I['G1'], axis=(-2, -1)) + np.sum(dm2 * I['G2'], axis=(-2, -1)))
    dG1 = -e[..., None, None] * dm1
    dG2 = -e[..., None, None] * dm2

    # omega: G_t = sum_{i in window(t)} g_i u_i  ->  du_i = g_i * R_i,
    # R_i = sum_{t=i}^{min(i+w-1, cs-1)} dG_t  (reverse windowed cumsum)
    def rev_window(dG):
        if omega <= 1:
            return dG
        return omega_aggregate(dG[:, ::-1], np.ones_like(dG[:, :1]), omega)[:, ::-1]
    if omega > 1:
        R1, R2 = rev_window(dG1), rev_window(dG2)
        dg = np.sum(R1 * I['u1'], axis=(-2, -1)) + np.sum(R2 * I['u2'], axis=(-2, -1))
        du1 = g[..., None, None] * R1
        du2 = g[..., None, None] * R2
    else:
        dg = np.zeros_like(g)
        du1, du2 = dG1, dG2

    # mem_grad: u1 = s err act^T ; u2 = s chain k^T ; chain = (W1^T err) * gp(h)
    derr = s * _ein('bchde,bche->bchd', du1, I['act'])
    dact = s * _ein('bchde,bchd->bche', du1, I['err'])
    dchain = s * _ein('bched,bchd->bche', du2, k)
    dk = s * _ein('bched,bche->bchd', du2, I['chain'])
    dw1t = dchain * I['gp']
    dh = dchain * I['w1t_err'] * gelu_erf_second(I['h']).astype(dt)
    dW1_in = dW1_in + _ein('bchd,bche->bhde', I['err'], dw1t)
    derr = derr + _ein('bhde,bche->bchd', W1, dw1t)

    # mem_fwd: err = k + W1 act - v ; act = gelu(h) ; h = W2 k
    dk = dk + derr
    dv = -derr
    dW1_in = dW1_in + _ein('bchd,bche->bhde', derr, I['act'])
    dact = dact + _ein('bhde,bchd->bche', W1, derr)
    dh = dh + dact * gelu_tanh_grad(I['h'])
    dW2_in = dW2_in + _ein('bche,bchd->bhed', dh, k)
    dk = dk + _ein('bhed,bche->bchd', W2, dh)

    grads = dict(q=dq, k=dk, v=dv, alpha=da, eta=de, theta=dth, gamma=dg)
    return grads, (dW1_in, dW2_in, dS1_in, dS2_in)


# ---------------------------------------------------------------------------
# full scan driver (memory_layer.py:649-718)
# ---------------------------------------------------------------------------

def lm_initial_state(B, H, D, E, dtype=np.float32):
    """atlas_jax/model.py:251-264: W1 = 0, W2 = [I; 0], S = 0."""
    W1 = np.zeros((B, H, D, E), dtype)
    W2 = np.zeros((B, H, E, D), dtype)
    m = min(D, E)
    W2[:, :, np.arange(m), np.arange(m)] = 1.0
    return (W1, W2, np.zeros((B, H, D, E), dtype), np.zeros((B, H, E, D), dtype))


def _pad(x, pad, value):
    if pad == 0:
        return x
    width = [(0, 0)] * x.ndim
    width[1] = (0, pad)
    return np.pad(x, width, constant_values=value)


def _prepare(q, k, v, alpha, eta, theta, gamma, chunk, dtype):
    T = q.shape[1]
    pad = (-T) % chunk
    cast = lambda x: np.asarray(x).astype(dtype)  # noqa: E731
    q, k, v = (_pad(cast(x), pad, 0.0) for x in (q, k, v))
    alpha = _pad(cast(alpha), pad, 1.0)                     # memory_layer.py:655
    eta = _pad(cast(eta), pad, 0.0)
    theta = _pad(cast(theta), pad, 0.0)
    # gamma=None means all ones, as a NULL gamma does at the C ABI (the reference
    # passes a gate only when omega > 1, memory_layer.py:435-438, 627-633)
    if gamma is None:
        gamma = np.ones(alpha.shape, dtype)
        gamma[:, T:] = 0.0
    else:
        gamma = _pad(cast(gamma), pad, 0.0)
    return T, q, k, v, alpha, eta, theta, gamma


def scan_forward(q, k, v, alpha, eta, theta, gamma, state, chunk=64, omega=16,
                 ns_steps=5, dtype=np.float32, return_carries=False):
    """Whole-sequence forward.  Returns (y (B,T,H,D), final_state[, carries]).

    ``carries[c]`` is the state entering chunk c (what the backward recomputes from)."""
    T, q, k, v, alpha, eta, theta, gamma = _prepare(q, k, v, alpha, eta, theta, gamma, chunk, dtype)
    st = tuple(np.asarray(x).astype(dtype) for x in state)
    n = q.shape[1] // chunk
    ys, carries = [], []
    for c in range(n):
        sl = slice(c * chunk, (c + 1) * chunk)
        carries.append(st)
        y_c, st = chunk_forward(st, q[:, sl], k[:, sl], v[:, sl], alpha[:, sl],
                                eta[:, sl], theta[:, sl], gamma[:, sl], omega, ns_steps)
        ys.append(y_c)
    y = np.concatenate(ys, axis=1)[:, :T]
    if return_carries:
        return y, st, carries
    return y, st


def scan_backward(q, k, v, alpha, eta, theta, gamma, state, dy, dstate=None,
                  chunk=64, omega=16, ns_steps=5, pe_ste=False,
                  stop_grad_chunks=False, dtype=np.float64):
    """VJP of ``scan_forward``.  Returns (grads dict, dstate_in tuple)."""
    T, q, k, v, alpha, eta, theta, gamma = _prepare(q, k, v, alpha, eta, theta, gamma, chunk, dtype)
    _, _, carries = scan_forward(q, k, v, alpha, eta, theta, gamma, state, chunk, omega,
                                 ns_steps, dtype, return_carries=True)
    dy = _pad(np.asarray(dy).astype(dtype), q.shape[1] - T, 0.0)
    if dstate is None:
        dst = tuple(np.zeros_like(x) for x in carries[0])
    else:
        dst = tuple(np.asarray(x).astype(dtype) for x in dstate)
    n = q.shape[1] // chunk
    out = {name: np.zeros_like(x) for name, x in
           dict(q=q, k=k, v=v, alpha=alpha, eta=eta, theta=theta, gamma=gamma).items()}
    for c in range(n - 1, -1, -1):
        sl = slice(c * chunk, (c + 1) * chunk)
        gr, dst = chunk_backward(carries[c], q[:, sl], k[:, sl], v[:, sl], alpha[:, sl],
                                 eta[:, sl], theta[:, sl], gamma[:, sl], dy[:, sl], dst,
                                 omega, ns_steps, pe_ste)
        for name, val in gr.items():
            out[name][:, sl] = val
        if stop_grad_chunks:
            dst = tuple(np.zeros_like(x) for x in dst)
    out = {name: val[:, :T] for name, val in out.items()}
    return out, dst


# ---------------------------------------------------------------------------
# synthetic inputs (BASELINE config distributions)
# ---------------------------------------------------------------------------

def _sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))


def make_inputs(B, T, H, D, seed=0, gamma_mode="ones"):
    """Seeded inputs: q,k,v ~ N(0,1) L2-normalised per head; alpha = sigmoid(N(3,.5)),
    eta = sigmoid(N(-3,.5)), theta = sigmoid(N(1,.5)); gamma = 1 ("ones") or
    sigmoid(N(0,.5)) ("random").  Draw order q, k, v, alpha, eta, theta, gamma."""
    rng = np.random.default_rng(seed)

    def unit(x):
        return x / np.linalg.norm(x, axis=-1, keepdims=True)
    q = unit(rng.standard_normal((B, T, H, D))).astype(np.float32)
    k = unit(rng.standard_normal((B, T, H, D))).astype(np.float32)
    v = unit(rng.standard_normal((B, T, H, D))).astype(np.float32)
    alpha = _sigmoid(rng.normal(3.0, 0.5, (B, T, H))).astype(np.float32)
    eta = _sigmoid(rng.normal(-3.0, 0.5, (B, T, H))).astype(np.float32)
    theta = _sigmoid(rng.normal(1.0, 0.5, (B, T, H))).astype(np.float32)
    if gamma_mode == "ones":
        gamma = np.ones((B, T, H), np.float32)
    else:
        gamma = _sigmoid(rng.normal(0.0, 0.5, (B, T, H))).astype(np.float32)
    return q, k, v, alpha, eta, theta, gamma


def make_xavier_state(B, H, D, E, seed=1, dtype=np.float32):
    """Standalone-layer initial state (memory_layer.py:448-452, 635-643): Xavier-uniform
    W1/W2 broadcast over B, S = 0."""
    rng = np.random.default_rng(seed)
    bound = math.sqrt(6.0 / (D + E))
    W1 = rng.uniform(-bound, bound, (H, D, E)).astype(dtype)
    W2 = rng.uniform(-bound, bound, (H, E, D)).astype(dtype)
    W1 = np.broadcast_to(W1, (B, H, D, E)).copy()
    W2 = np.broadcast_to(W2, (B, H, E, D)).copy()
    return (W1, W2, np.zeros((B, H, D, E), dtype), np.zeros((B, H, E, D), dtype))


# ----------------------------------------------------------------------------
# Layer prologue / epilogue around the scan (memory_layer.py:606-633, 720-722)
# ----------------------------------------------------------------------------
def rms_norm(x):
    """memory_layer.py:211-216 (mean of squares over the last axis, eps 1e-6)."""
    return x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + 1e-6)


def short_conv(x, w, b):
    """Causal depthwise conv, memory_layer.py:303-329.  x (B,T,C), w (C,K), b (C)."""
    K = w.shape[-1]
    xp = np.concatenate([np.zeros((x.shape[0], K - 1, x.shape[2]), x.dtype), x], axis=1)
    out = np.broadcast_to(b, x.shape).astype(x.dtype).copy()
    for j in range(K):
        out += w[:, j] * xp[:, j:j + x.shape[1]]
    return out


def poly_features(x, a):
    """memory_layer.py:455-462: sum_i a_i x^(i+1)."""
    out, xp = a[0] * x, x
    for i in range(1, len(a)):
        xp = xp * x
        out = out + a[i] * xp
    return out


def layer_prologue(proj, B, T, H, D, conv_w, conv_b, poly, gate_bias, has_gamma, has_retrieve, max_lr):
    """memory_layer.py:606-633 (and the retrieve gate's sigmoid, 720-721) applied to the
    concatenated projection proj (B*T, 3*H*D + G*H), columns [q|k|v|alpha|eta|theta|gamma?|retrieve?].
    Returns q, k, v (B,T,H,D) and the activated gates [alpha, eta, theta, gamma|None, retrieve|None]."""
    di = H * D
    P = proj.reshape(B, T, -1)
    qkv = [short_conv(P[..., i * di:(i + 1) * di], conv_w[i], conv_b[i]).reshape(B, T, H, D) for i in range(3)]
    q, k, v = qkv
    if poly is not None and len(poly) > 0:
        q = poly_features(rms_norm(q), poly)
        k = rms_norm(poly_features(k, poly))
    else:
        q, k = rms_norm(q), rms_norm(k)
    names = ["alpha", "eta", "theta"] + (["gamma"] if has_gamma else []) + (["retrieve"] if has_retrieve else [])
    gates = {}
    for i, n in enumerate(names):
        z = P[..., 3 * di + i * H:3 * di + (i + 1) * H]
        if n != "retrieve":
            z = z + gate_bias[i]
        s = _sigmoid(z)
        gates[n] = s * max_lr if n == "eta" else s
    return q, k, v, [gates.get(n) for n in ("alpha", "eta", "theta", "gamma", "retrieve")]
