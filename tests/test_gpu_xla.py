"""GPU check of the XLA custom-call adapters (atlas_xla_fwd / atlas_xla_bwd): the
buffer array a JAX registration passes (operands then results, the packed
AtlasScanParams as opaque) must give exactly what atlas_scan_fwd / atlas_scan_bwd
give on the same inputs.  The forward is deterministic, so it is compared bit for
bit.  The backward forms its gate gradients and frozen-pass sums with atomics whose
order varies between runs, and the scan's cotangents amplify such rounding
differences, so two runs of atlas_scan_bwd itself differ slightly; the adapter is
held to the north-star tolerance against it (1e-4 relative in fp32, 2e-2 in bf16)."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import atlas_oracle as O
from gpu_util import rel, to_dev, to_np

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("act", [torch.float32, torch.bfloat16])
def test_xla_adapters_match_the_c_abi(act):
    from atlas_b200 import _lib as L
    from atlas_b200 import ScanConfig, ATLAS_PREC_TENSOR, scan_forward, scan_backward
    from atlas_b200.scan import _params
    lib = L.load()
    B, T, H, D, E = 1, 64, 2, 64, 256
    cfg = ScanConfig(chunk=64, omega=16, ns_steps=5, precision=ATLAS_PREC_TENSOR)
    q, k, v, a, e, t, g = O.make_inputs(B, T, H, D, seed=21, gamma_mode="random")
    st = O.make_xavier_state(B, H, D, E, seed=22)
    st = (st[0], st[1], 0.05 * st[0], 0.05 * st[1])
    ins = [to_dev(q, act), to_dev(k, act), to_dev(v, act), to_dev(a), to_dev(e), to_dev(t), to_dev(g)]
    state = [to_dev(x) for x in st]
    y_ref, out_ref, saved_ref = scan_forward(*ins, tuple(state), cfg)

    p = _params(cfg, B, T, H, D, E, act)
    opaque = ctypes.string_at(ctypes.byref(p), ctypes.sizeof(p))
    dev = ins[0].device
    y = torch.empty_like(ins[0])
    out = [torch.empty_like(x) for x in state]
    saved = torch.empty(lib.atlas_scan_saved_bytes(ctypes.byref(p)), dtype=torch.uint8, device=dev)
    ws = torch.empty(lib.atlas_scan_workspace_bytes(ctypes.byref(p)), dtype=torch.uint8, device=dev)
    bufs = ins + state + [y] + out + [saved, ws]
    arr = (ctypes.c_void_p * len(bufs))(*[x.data_ptr() for x in bufs])
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    lib.atlas_xla_fwd(stream, arr, opaque, len(opaque), None)
    torch.cuda.synchronize()
    assert lib.atlas_last_error_string() == b""
    assert torch.equal(y, y_ref)
    for x, r in zip(out, out_ref):
        assert torch.equal(x, r)
    assert torch.equal(saved, saved_ref)

    rng = np.random.default_rng(23)
    dy = to_dev(rng.standard_normal((B, T, H, D)).astype(np.float32), act)
    dfin = [to_dev(0.1 * rng.standard_normal(x.shape).astype(np.float32)) for x in st]
    ref = scan_backward(*ins, saved_ref, dy, tuple(dfin), cfg, E)
    grads = [torch.empty_like(x) for x in ins[:3]] + [torch.empty_like(x) for x in ins[3:]]
    dstate = [torch.empty_like(x) for x in state]
    ws2 = torch.empty_like(ws)
    bufs = ins + [saved, dy] + dfin + grads + dstate + [ws2]
    arr = (ctypes.c_void_p * len(bufs))(*[x.data_ptr() for x in bufs])
    lib.atlas_xla_bwd(stream, arr, opaque, len(opaque), None)
    torch.cuda.synchronize()
    assert lib.atlas_last_error_string() == b""
    for x, r in zip(grads + dstate, list(ref[:7]) + list(ref[7])):
        assert rel(to_np(x), to_np(r)) <= (1e-4 if act == torch.float32 else 2e-2)


def test_xla_polar_express_matches_the_c_abi():
    """atlas_xla_polar_express (the Muon target, opaque packed as the JAX binding
    packs it) gives what atlas_polar_express_batched gives, bit for bit."""
    import struct
    from atlas_b200 import _lib as L
    from atlas_b200 import polar_express
    lib = L.load()
    g = torch.Generator(device="cuda").manual_seed(5)
    X = torch.randn(3, 768, 256, device="cuda", generator=g)
    ref = polar_express(X, steps=5, eps_in_sqrt=0.0, precision=L.ATLAS_PREC_TENSOR)
    Y = torch.empty_like(X)
    ws = torch.empty(lib.atlas_polar_express_workspace_bytes(3, 768, 256, 5, L.ATLAS_PREC_TENSOR),
                     dtype=torch.uint8, device="cuda")
    opaque = struct.pack("<qiiiifi", 3, 768, 256, 5, L.ATLAS_PREC_TENSOR, 0.0, 0)
    arr = (ctypes.c_void_p * 3)(X.data_ptr(), Y.data_ptr(), ws.data_ptr())
    lib.atlas_xla_polar_express(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), arr, opaque,
                                len(opaque), None)
    torch.cuda.synchronize()
    assert lib.atlas_last_error_string() == b""
    assert torch.equal(Y, ref)
