"""GPU test of atlas_scan_fwd_noalloc, the forward entry point that allocates
nothing.  It exists for callers that cannot call cudaMalloc, for example code
that runs inside a memory allocator or an inference runtime that forbids device
allocations once it has started; such callers cannot provide the workspace the
regular entry point asks for.  The test calls it twice in a row through the
C ABI, on different inputs, and compares both results with atlas_scan_fwd
(tolerance 2e-2 relative, the tensor path's bound; the two share the kernel, so
the results normally match exactly).  This file sorts last so that a run that
stops at the first failure has already run every other test."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import atlas_oracle as O
from gpu_util import rel, to_dev, to_np

pytestmark = pytest.mark.gpu
TOL = 2e-2


def _noalloc(lib, L, p, ins, st):
    B, T, H, D = ins[0].shape
    E = 256
    y = torch.empty_like(ins[0])
    out = [torch.empty(B, H, D, E, device="cuda"), torch.empty(B, H, E, D, device="cuda"),
           torch.empty(B, H, D, E, device="cuda"), torch.empty(B, H, E, D, device="cuda")]
    P = lambda t: None if t is None else ctypes.c_void_p(t.data_ptr())  # noqa: E731
    stv = [None] * 4 if st is None else [P(x) for x in st]
    rc = lib.atlas_scan_fwd_noalloc(ctypes.byref(p), *[P(x) for x in ins], *stv, P(y), *[P(x) for x in out],
                                    ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    L.check(rc)
    return y, out


def test_noalloc_forward_matches_regular_forward_twice():
    from atlas_b200 import _lib as L
    from atlas_b200 import ScanConfig, ATLAS_PREC_TENSOR, scan_forward, device_status
    lib = L.load()
    B, T, H, D, E = 2, 130, 4, 64, 256
    cfg = ScanConfig(chunk=64, omega=16, ns_steps=5, precision=ATLAS_PREC_TENSOR)
    p = L.AtlasScanParams(L.ATLAS_ABI_VERSION, B, T, H, D, E, 64, 16, 5, 0, 0, L.ATLAS_BF16, L.ATLAS_PREC_TENSOR)
    for call, seed in enumerate((21, 22)):
        q, k, v, a, e, t, g = O.make_inputs(B, T, H, D, seed=seed, gamma_mode="random")
        ins = [to_dev(q, torch.bfloat16), to_dev(k, torch.bfloat16), to_dev(v, torch.bfloat16),
               to_dev(a), to_dev(e), to_dev(t), to_dev(g)]
        st = None
        if call == 1:  # second call also passes an explicit initial state
            s0 = O.make_xavier_state(B, H, D, E, seed=seed)
            st = [to_dev(x) for x in (s0[0], s0[1], 0.05 * s0[0], 0.05 * s0[1])]
        if call == 1:  # same call once first, so that lazily loaded kernels are resident
            _noalloc(lib, L, p, ins, st)
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        y_n, out_n = _noalloc(lib, L, p, ins, st)
        torch.cuda.synchronize()
        free1 = torch.cuda.mem_get_info()[0]
        if call == 1:  # the call itself must not take device memory
            assert free1 == free0, (free0, free1)
        y_r, out_r, _ = scan_forward(*ins, st, cfg, need_saved=True)
        torch.cuda.synchronize()
        device_status()
        assert rel(to_np(y_n), to_np(y_r)) < TOL
        for i, (x_n, x_r) in enumerate(zip(out_n, out_r)):
            r, n = to_np(x_r), to_np(x_n)
            if i < 2:  # W1, W2 are non-zero on these inputs
                assert r.any()
            if r.any():
                assert rel(n, r) < TOL
            else:  # the momentum leaves the padded last chunk at zero (theta = 0 on padding)
                assert not n.any()


def test_noalloc_rejects_too_many_chains():
    from atlas_b200 import _lib as L
    lib = L.load()
    p = L.AtlasScanParams(L.ATLAS_ABI_VERSION, 4, 64, 8, 64, 256, 64, 16, 5, 0, 0, L.ATLAS_BF16, L.ATLAS_PREC_TENSOR)
    dummy = torch.empty(16, device="cuda")
    ptr = ctypes.c_void_p(dummy.data_ptr())
    rc = lib.atlas_scan_fwd_noalloc(ctypes.byref(p), ptr, ptr, ptr, ptr, ptr, ptr, None, None, None, None, None,
                                    ptr, None, None, None, None, None)
    assert rc == L.ATLAS_ERR_INVALID_ARGUMENT
    assert b"ATLAS_NOALLOC_MAX_CHAINS" in lib.atlas_last_error_string()
