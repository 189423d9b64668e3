"""GPU parity of the tcgen05 backward scan against the oracle's float64 VJP.

Tolerance per gradient tensor: 2e-2 relative (Frobenius) with bf16 activations
(inputs rounded to bf16 for both sides); with float32 activations
max(2e-4, 2 x the float32 oracle VJP's own distance from the float64 one)
(gpu_util.f32_bound_bwd): the reference's float32 accuracy up to the summation
order of the scalar gate gradients.
"""
import numpy as np
import pytest
import torch

from oracle import atlas_oracle as O
from gpu_util import check_errs, f32_bound_bwd, rel, to_dev, to_np

pytestmark = pytest.mark.gpu
TOL = 2e-2


def _bf(x):
    import ml_dtypes
    return x.astype(ml_dtypes.bfloat16).astype(np.float32)


@pytest.mark.parametrize("T,omega,ste,sg,act,xav", [
    (128, 16, False, False, torch.float32, False),
    (100, 4, False, False, torch.bfloat16, True),
    (128, 16, True, False, torch.float32, True),
    (128, 8, False, True, torch.float32, True),
])
def test_tc_backward(T, omega, ste, sg, act, xav):
    from atlas_b200 import ScanConfig, ATLAS_PREC_TENSOR, scan_forward, scan_backward, device_status
    B, H, D, E, cs = 1, 2, 64, 256, 64
    ins = O.make_inputs(B, T, H, D, seed=11, gamma_mode="random")
    if act == torch.bfloat16:
        ins = tuple(_bf(x) for x in ins[:3]) + tuple(ins[3:])
    if xav:
        st = O.make_xavier_state(B, H, D, E, seed=12)
        st = (st[0], st[1], 0.05 * st[0], 0.05 * st[1])
    else:
        st = O.lm_initial_state(B, H, D, E)
    cfg = ScanConfig(chunk=cs, omega=omega, ns_steps=5, pe_ste=ste, stop_grad_chunks=sg,
                     precision=ATLAS_PREC_TENSOR)
    q, k, v, a, e, t, g = ins
    dev_in = [to_dev(q, act), to_dev(k, act), to_dev(v, act), to_dev(a), to_dev(e), to_dev(t), to_dev(g)]
    y, out, saved = scan_forward(*dev_in, tuple(to_dev(x) for x in st), cfg)
    rng = np.random.default_rng(13)
    dy = rng.standard_normal((B, T, H, D)).astype(np.float32)
    if act == torch.bfloat16:
        dy = _bf(dy)
    dfin = [0.1 * rng.standard_normal(x.shape).astype(np.float32) for x in st]
    res = scan_backward(*dev_in, saved, to_dev(dy, act), tuple(to_dev(x) for x in dfin), cfg, E)
    torch.cuda.synchronize()
    device_status()
    grads, dst = O.scan_backward(*ins, st, dy, dfin, cs, omega, 5, pe_ste=ste, stop_grad_chunks=sg)
    if act == torch.float32:
        g32, d32 = O.scan_backward(*ins, st, dy, dfin, cs, omega, 5, pe_ste=ste, stop_grad_chunks=sg,
                                   dtype=np.float32)
    errs, bounds = {}, {}
    for name, val in zip(("q", "k", "v", "alpha", "eta", "theta", "gamma"), res[:7]):
        errs[name] = rel(to_np(val), grads[name])
        bounds[name] = TOL if act == torch.bfloat16 else f32_bound_bwd(g32[name], grads[name])
    for i, n in enumerate(("dW1", "dW2", "dS1", "dS2")):
        if np.abs(dst[i]).max() > 0:
            errs[n] = rel(to_np(res[7][i]), dst[i])
            bounds[n] = TOL if act == torch.bfloat16 else f32_bound_bwd(d32[i], dst[i])
    check_errs(errs, bounds)


@pytest.mark.parametrize("T,chunk,omega,ns", [(40, 32, 64, 5), (64, 64, 16, 2), (1, 64, 16, 5)])
def test_tc_backward_edge_cases(T, chunk, omega, ns):
    from atlas_b200 import ScanConfig, ATLAS_PREC_TENSOR, scan_forward, scan_backward
    B, H, D, E = 1, 2, 64, 256
    ins = O.make_inputs(B, T, H, D, seed=40 + T, gamma_mode="random")
    st = O.make_xavier_state(B, H, D, E, seed=41)
    st = (st[0], st[1], 0.05 * st[0], 0.05 * st[1])
    cfg = ScanConfig(chunk=chunk, omega=omega, ns_steps=ns, precision=ATLAS_PREC_TENSOR)
    q, k, v, a, e, t, g = ins
    dev = [to_dev(x) for x in ins]
    y, out, saved = scan_forward(*dev, tuple(to_dev(x) for x in st), cfg)
    dy = np.random.default_rng(3).standard_normal((B, T, H, D)).astype(np.float32)
    res = scan_backward(*dev, saved, to_dev(dy), None, cfg, E)
    torch.cuda.synchronize()
    grads, dst = O.scan_backward(*ins, st, dy, None, chunk, omega, ns)
    g32, d32 = O.scan_backward(*ins, st, dy, None, chunk, omega, ns, dtype=np.float32)
    names = ("q", "k", "v", "alpha", "eta", "theta", "gamma")
    errs = {n: rel(to_np(v_), grads[n]) for n, v_ in zip(names, res[:7])}
    bounds = {n: f32_bound_bwd(g32[n], grads[n]) for n in names}
    for i, n in enumerate(("dW1", "dW2", "dS1", "dS2")):
        if np.abs(dst[i]).max() > 0:
            errs[n], bounds[n] = rel(to_np(res[7][i]), dst[i]), f32_bound_bwd(d32[i], dst[i])
    check_errs(errs, bounds)
