"""GPU parity of the shape-generic batched tensor-path forward (scan_gen.cu):
head_dim 128 with memory width 512 (the long-context sweep's state split case),
chunk 128, D == E (the Pallas kernel's regime, pallas_fused.py:36-311), the default
170M shape through the batched path, many chains, and the linear-memory variant
(memory_layer.py:468-494).

Tolerances as for the fused path: 2e-2 relative with bf16 activations; with float32
activations max(1e-4, 1.5 x the float32 oracle's own error) (gpu_util.f32_bound)."""
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


def _deep(B, T, H, D, E, chunk, omega, ns, act, xavier, seed, precision=None):
    from atlas_b200 import ScanConfig, ATLAS_PREC_TENSOR_BATCHED, scan_forward, device_status
    ins = O.make_inputs(B, T, H, D, seed=seed, gamma_mode="random")
    if act == torch.bfloat16:
        ins = tuple(_bf(x) for x in ins[:3]) + tuple(ins[3:])
    if xavier:
        st = O.make_xavier_state(B, H, D, E, seed=seed + 1)
        st = (st[0], st[1], 0.05 * st[0], 0.05 * st[1])
    else:
        st = O.lm_initial_state(B, H, D, E)
    cfg = ScanConfig(chunk=chunk, omega=omega, ns_steps=ns,
                     precision=ATLAS_PREC_TENSOR_BATCHED if precision is None else precision)
    q, k, v, a, e, t, g = ins
    y, out, _ = scan_forward(to_dev(q, act), to_dev(k, act), to_dev(v, act), to_dev(a), to_dev(e), to_dev(t),
                             to_dev(g), tuple(to_dev(x) for x in st) if xavier else None, cfg)
    torch.cuda.synchronize()
    device_status()
    y_o, fin = O.scan_forward(*ins, st, chunk, omega, ns, dtype=np.float64)
    names = ("y", "W1", "W2", "S1", "S2")
    got = [to_np(y)] + [to_np(x) for x in out]
    ref = [y_o] + list(fin)
    errs, bounds = {}, {}
    if act == torch.float32:
        y32, fin32 = O.scan_forward(*ins, st, chunk, omega, ns, dtype=np.float32)
        r32 = [y32] + list(fin32)
    for i, n in enumerate(names):
        if np.abs(ref[i]).max() == 0:
            assert np.all(got[i] == 0), n
            continue
        errs[n] = rel(got[i], ref[i])
        bounds[n] = TOL if act == torch.bfloat16 else f32_bound(r32[i], ref[i])
    check_errs(errs, bounds)


@pytest.mark.parametrize("act", [torch.float32, torch.bfloat16])
def test_batched_head_dim_128_chunk_128(act):
    """Config 4's state-split case: D=128, E=512 (1 MB of float32 state per chain), chunk 128, padding."""
    _deep(1, 200, 1, 128, 512, 128, 16, 5, act, xavier=True, seed=1)


def test_batched_default_shape_matches_oracle():
    """The 170M layer shape through the batched path, LM initial state, padding."""
    _deep(1, 150, 2, 64, 256, 64, 16, 5, torch.float32, xavier=False, seed=2)


@pytest.mark.parametrize("D,E,chunk,omega", [(64, 64, 32, 8), (32, 32, 64, 4), (32, 128, 128, 64)])
def test_batched_d_equals_e_and_chunk_sizes(D, E, chunk, omega):
    """D == E (pallas_fused.py's regime), chunk 32/64/128, Omega >= chunk."""
    _deep(2, 140, 1, D, E, chunk, omega, 5, torch.float32, xavier=True, seed=D + E + chunk)


def test_tensor_precision_routes_other_shapes_to_the_batched_forward():
    """ATLAS_PREC_TENSOR with D=128 runs the batched forward (the fused kernels cover
    D=64, E=256, chunk <= 64 only); fewer Newton-Schulz steps."""
    from atlas_b200 import ATLAS_PREC_TENSOR
    _deep(1, 64, 2, 128, 512, 64, 8, 3, torch.float32, xavier=True, seed=7, precision=ATLAS_PREC_TENSOR)


def test_batched_many_chains_bf16():
    """48 chains in one launch (bf16 q/k/v)."""
    _deep(4, 64, 12, 64, 256, 64, 16, 5, torch.bfloat16, xavier=False, seed=9)


@pytest.mark.parametrize("act,D,chunk,omega,T", [(torch.float32, 64, 64, 16, 130), (torch.bfloat16, 64, 64, 16, 130),
                                                 (torch.float32, 32, 32, 1, 70), (torch.float32, 128, 128, 64, 150)])
def test_linear_memory_forward(act, D, chunk, omega, T):
    """Linear memory (deep_memory=False): zero initial state and a random one."""
    from atlas_b200 import ScanConfig, ATLAS_PREC_TENSOR, linear_scan_forward, device_status
    B, H = 2, 2
    ins = O.make_inputs(B, T, H, D, seed=D + T, gamma_mode="random")
    if act == torch.bfloat16:
        ins = tuple(_bf(x) for x in ins[:3]) + tuple(ins[3:])
    cfg = ScanConfig(chunk=chunk, omega=omega, ns_steps=5, precision=ATLAS_PREC_TENSOR)
    rng = np.random.default_rng(3)
    for st in (None, (0.1 * rng.standard_normal((B, H, D, D)).astype(np.float32),
                      0.01 * rng.standard_normal((B, H, D, D)).astype(np.float32))):
        q, k, v, a, e, t, g = ins
        y, out = linear_scan_forward(to_dev(q, act), to_dev(k, act), to_dev(v, act), to_dev(a), to_dev(e),
                                     to_dev(t), to_dev(g), None if st is None else tuple(to_dev(x) for x in st),
                                     cfg)
        torch.cuda.synchronize()
        device_status()
        y_o, fin = O.scan_forward_linear(*ins, st, chunk, omega, 5, dtype=np.float64)
        errs = {"y": rel(to_np(y), y_o), "M": rel(to_np(out[0]), fin[0])}
        if np.abs(fin[1]).max() > 0:
            errs["S"] = rel(to_np(out[1]), fin[1])
        if act == torch.bfloat16:
            bounds = dict.fromkeys(errs, TOL)
        else:
            y32, f32 = O.scan_forward_linear(*ins, st, chunk, omega, 5, dtype=np.float32)
            r32 = {"y": (y32, y_o), "M": (f32[0], fin[0]), "S": (f32[1], fin[1])}
            bounds = {n: f32_bound(*r32[n]) for n in errs}
        check_errs(errs, bounds)


def test_forward_only_few_chains_takes_the_batched_forward():
    """A forward-only ATLAS_PREC_TENSOR call (no saved carries) with few chains runs the
    batched forward (as ATLAS_PREC_TENSOR_BATCHED does); with saved carries it stays
    on the fused kernels the backward needs.  Both match the oracle."""
    import numpy as np
    from atlas_b200 import ATLAS_PREC_TENSOR, ATLAS_PREC_TENSOR_BATCHED, ScanConfig, scan_forward
    B, T, H = 2, 150, 3
    ins = O.make_inputs(B, T, H, 64, seed=21)
    dev = [to_dev(x) for x in ins]
    res = {}
    for name, prec, keep in (("auto", ATLAS_PREC_TENSOR, False), ("batched", ATLAS_PREC_TENSOR_BATCHED, False),
                             ("fused", ATLAS_PREC_TENSOR, True)):
        cfg = ScanConfig(chunk=64, omega=16, ns_steps=5, precision=prec)
        y, out, saved = scan_forward(*dev, None, cfg, need_saved=keep)
        torch.cuda.synchronize()
        res[name] = to_np(y)
    # the batched read-out sums with float atomics, so two batched runs agree to rounding
    # only; the fused kernels differ from it by far more than that
    d_batched, d_fused = rel(res["auto"], res["batched"]), rel(res["auto"], res["fused"])
    print(f"auto vs batched {d_batched:.2e}, auto vs fused {d_fused:.2e}")
    assert d_batched < 1e-6 and d_batched < 0.1 * d_fused
    y_o, _ = O.scan_forward(*ins, O.lm_initial_state(B, H, 64, 256), 64, 16, 5, dtype=np.float64)
    y32, _ = O.scan_forward(*ins, O.lm_initial_state(B, H, 64, 256), 64, 16, 5, dtype=np.float32)
    for name in ("auto", "fused"):
        assert rel(res[name], y_o) <= f32_bound(y32, y_o), name
