"""Failure detection without a GPU fault: the tensor path's chunk-ordering waits
are bounded.  With the test hook raising the wait threshold to a value nothing
ever writes, a launch must end by itself and report ATLAS_ERR_DEVICE_TIMEOUT
through the status word, and the context must stay usable afterwards."""
import numpy as np
import pytest
import torch

from oracle import atlas_oracle as O
from gpu_util import rel, to_dev, to_np

pytestmark = pytest.mark.gpu


def _inputs():
    q, k, v, a, e, t, g = O.make_inputs(1, 128, 2, 64, seed=31, gamma_mode="random")  # 2 chunks
    return [to_dev(q, torch.bfloat16), to_dev(k, torch.bfloat16), to_dev(v, torch.bfloat16),
            to_dev(a), to_dev(e), to_dev(t), to_dev(g)]


def test_bounded_wait_reports_timeout_and_context_survives():
    from atlas_b200 import _lib as L
    from atlas_b200 import ScanConfig, ATLAS_PREC_TENSOR, scan_forward, scan_backward
    lib = L.load()
    cfg = ScanConfig(chunk=64, omega=16, ns_steps=5, precision=ATLAS_PREC_TENSOR)
    ins = _inputs()
    y_ref, _, saved = scan_forward(*ins, None, cfg)
    torch.cuda.synchronize()
    assert lib.atlas_scan_status() == L.ATLAS_OK
    try:
        lib.atlas_debug_set_wait_hooks(1000, 20000)        # a flag value nothing sets
        scan_forward(*ins, None, cfg)
        torch.cuda.synchronize()
        assert lib.atlas_scan_status() == L.ATLAS_ERR_DEVICE_TIMEOUT
        dy = torch.ones_like(ins[0])
        scan_backward(*ins, saved, dy, None, cfg, 256)
        torch.cuda.synchronize()
        assert lib.atlas_scan_status() == L.ATLAS_ERR_DEVICE_TIMEOUT
    finally:
        lib.atlas_debug_set_wait_hooks(0, 0)
    y2, _, _ = scan_forward(*ins, None, cfg)              # the context is still usable
    torch.cuda.synchronize()
    assert lib.atlas_scan_status() == L.ATLAS_OK
    assert rel(to_np(y2), to_np(y_ref)) == 0.0             # and the kernel is deterministic
