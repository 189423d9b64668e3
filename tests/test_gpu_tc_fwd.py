"""GPU parity of the tcgen05 forward scan against the oracle.

Tolerances (north_star): 2e-2 relative (Frobenius) with bf16 activations; with
float32 activations every output must be as close to the float64 oracle as
max(1e-4, 1.5 x the float32 oracle's own distance from it) -- the accuracy of the
reference's float32 arithmetic (gpu_util.f32_bound).  The oracle runs on the same
(bf16-rounded where applicable) inputs.
"""
import numpy as np
import pytest
import torch

from oracle import atlas_oracle as O
from gpu_util import check_errs, f32_bound, rel, to_dev, to_np

pytestmark = pytest.mark.gpu
TOL = 2e-2


def _bf(x):
    import ml_dtypes
    return x.astype(ml_dtypes.bfloat16).astype(np.float32)


def _run(ins, st, act, chunk=64, omega=16):
    from atlas_b200 import ScanConfig, ATLAS_PREC_TENSOR, scan_forward
    cfg = ScanConfig(chunk=chunk, omega=omega, ns_steps=5, precision=ATLAS_PREC_TENSOR)
    q, k, v, a, e, t, g = ins
    state = None if st is None else tuple(to_dev(x) for x in st)
    y, out, saved = scan_forward(to_dev(q, act), to_dev(k, act), to_dev(v, act), to_dev(a), to_dev(e), to_dev(t),
                                 to_dev(g), state, cfg)
    torch.cuda.synchronize()
    from atlas_b200 import device_status
    device_status()
    return to_np(y), [to_np(x) for x in out]


@pytest.mark.parametrize("act", [torch.bfloat16, torch.float32])
def test_tc_forward_lm_init(act):
    B, T, H = 1, 256, 2
    ins = O.make_inputs(B, T, H, 64, seed=0)
    if act == torch.bfloat16:
        ins = tuple(_bf(x) for x in ins[:3]) + tuple(ins[3:])
    y, out = _run(ins, None, act)
    st0 = O.lm_initial_state(B, H, 64, 256)
    y_o, fin = O.scan_forward(*ins, st0, 64, 16, 5, dtype=np.float64)
    names = ("y", "W1", "W2", "S1", "S2")
    errs = dict(zip(names, [rel(y, y_o)] + [rel(a, b) for a, b in zip(out, fin)]))
    if act == torch.bfloat16:
        bounds = dict.fromkeys(names, TOL)
    else:
        y32, fin32 = O.scan_forward(*ins, st0, 64, 16, 5, dtype=np.float32)
        bounds = dict(zip(names, [f32_bound(y32, y_o)] + [f32_bound(a, b) for a, b in zip(fin32, fin)]))
    check_errs(errs, bounds)


def test_tc_forward_padding_xavier_random_gamma():
    B, T, H = 2, 200, 1
    ins = O.make_inputs(B, T, H, 64, seed=3, gamma_mode="random")
    st = O.make_xavier_state(B, H, 64, 256, seed=4)
    st = (st[0], st[1], 0.05 * st[0], 0.05 * st[1])
    y, out = _run(ins, st, torch.float32, omega=4)
    y_o, fin = O.scan_forward(*ins, st, 64, 4, 5, dtype=np.float64)
    y32, fin32 = O.scan_forward(*ins, st, 64, 4, 5, dtype=np.float32)
    errs = {"y": rel(y, y_o), "W1": rel(out[0], fin[0]), "W2": rel(out[1], fin[1])}
    check_errs(errs, {"y": f32_bound(y32, y_o), "W1": f32_bound(fin32[0], fin[0]),
                      "W2": f32_bound(fin32[1], fin[1])})
    assert np.all(out[2] == 0) and np.all(out[3] == 0)  # padded tail zeroes S (memory_layer.py:657)


def test_tc_forward_many_chains_migrate_between_clusters():
    """96 chains (the 170M config's B*H per GPU) exceed the resident clusters, so
    chunks of one chain run on different clusters."""
    B, T, H = 8, 128, 12
    ins = O.make_inputs(B, T, H, 64, seed=5)
    ins = tuple(_bf(x) for x in ins[:3]) + tuple(ins[3:])
    y, out = _run(ins, None, torch.bfloat16)
    y_o, fin = O.scan_forward(*ins, O.lm_initial_state(B, H, 64, 256), 64, 16, 5, dtype=np.float64)
    errs = [rel(y, y_o)] + [rel(a, b) for a, b in zip(out, fin)]
    print("rel errors:", errs)
    assert max(errs) < TOL, errs


@pytest.mark.parametrize("T,chunk,omega,ns", [(1, 64, 16, 5), (96, 32, 8, 5), (128, 32, 64, 5), (70, 64, 16, 1),
                                              (64, 64, 16, 3), (130, 16, 4, 5), (300, 128, 16, 5),
                                              (256, 128, 128, 5), (129, 128, 8, 2), (100, 96, 16, 5)])
def test_tc_forward_edge_cases(T, chunk, omega, ns):
    """single token, chunk 32 / 16 / 128 / 96 (BASELINE sweep chunks; chunks above 64 run
    their frozen pass in 64-token parts), Omega >= chunk (full in-chunk cumsum,
    memory_layer.py:247-248), fewer Newton-Schulz steps."""
    from atlas_b200 import ScanConfig, ATLAS_PREC_TENSOR, scan_forward
    B, H = 1, 2
    ins = O.make_inputs(B, T, H, 64, seed=T + chunk, gamma_mode="random")
    st = O.make_xavier_state(B, H, 64, 256, seed=5)
    st = (st[0], st[1], 0.05 * st[0], 0.05 * st[1])
    cfg = ScanConfig(chunk=chunk, omega=omega, ns_steps=ns, precision=ATLAS_PREC_TENSOR)
    q, k, v, a, e, t, g = ins
    y, out, _ = scan_forward(to_dev(q), to_dev(k), to_dev(v), to_dev(a), to_dev(e), to_dev(t), to_dev(g),
                             tuple(to_dev(x) for x in st), cfg)
    torch.cuda.synchronize()
    y_o, fin = O.scan_forward(*ins, st, chunk, omega, ns, dtype=np.float64)
    y32, fin32 = O.scan_forward(*ins, st, chunk, omega, ns, dtype=np.float32)
    errs, bounds = {"y": rel(to_np(y), y_o)}, {"y": f32_bound(y32, y_o)}
    for i, (a_, b_, c_) in enumerate(zip(out, fin, fin32)):
        if np.abs(b_).max() > 0:
            errs[f"state{i}"], bounds[f"state{i}"] = rel(to_np(a_), b_), f32_bound(c_, b_)
    check_errs(errs, bounds)


def test_tc_forward_sweep_384_chains():
    """BASELINE config 4's largest B*H (384 (b,h) pairs) in one launch: four chains
    per resident cluster, chunks migrating between clusters."""
    B, T, H = 32, 64, 12
    ins = O.make_inputs(B, T, H, 64, seed=9)
    ins = tuple(_bf(x) for x in ins[:3]) + tuple(ins[3:])
    y, out = _run(ins, None, torch.bfloat16)
    y_o, fin = O.scan_forward(*ins, O.lm_initial_state(B, H, 64, 256), 64, 16, 5, dtype=np.float64)
    errs = [rel(y, y_o)] + [rel(a, b) for a, b in zip(out[:2], fin[:2])]
    assert max(errs) < TOL, errs


def test_tc_forward_chunk_128_many_chains():
    """Config 4's chunk 128 on the fused forward: 96 chains, bf16, chunks migrating
    between clusters, a padded last chunk."""
    B, T, H = 8, 320, 12
    ins = O.make_inputs(B, T, H, 64, seed=11)
    ins = tuple(_bf(x) for x in ins[:3]) + tuple(ins[3:])
    y, out = _run(ins, None, torch.bfloat16, chunk=128)
    y_o, fin = O.scan_forward(*ins, O.lm_initial_state(B, H, 64, 256), 128, 16, 5, dtype=np.float64)
    errs = [rel(y, y_o)] + [rel(a, b) for a, b in zip(out, fin)]
    print("rel errors:", errs)
    assert max(errs) < TOL, errs
