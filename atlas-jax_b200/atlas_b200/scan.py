"""Host-side API of the Atlas scan over the C ABI.

Torch is used only for device memory and the current CUDA stream; every
computation happens in libatlas_scan.so.  The functions mirror the reference's
boundary (atlas_jax/memory_layer.py:635-718 for the scan, fused_chunk.py:321-379
for the custom-VJP pair): ``scan_forward`` / ``scan_backward`` are the two halves
of the custom VJP and ``AtlasScan`` glues them into autograd.
"""

import ctypes
from dataclasses import dataclass

import torch

from . import _lib as L


@dataclass(frozen=True)
class ScanConfig:
    chunk: int = 64            # config.py:14
    omega: int = 16            # config.py:17
    ns_steps: int = 5          # config.py:16
    pe_ste: bool = False       # config.py:21
    stop_grad_chunks: bool = False  # config.py:29
    precision: int = L.ATLAS_PREC_TENSOR


def _params(cfg, B, T, H, D, E, act_dtype):
    return L.AtlasScanParams(L.ATLAS_ABI_VERSION, B, T, H, D, E, cfg.chunk, cfg.omega, cfg.ns_steps,
                             int(cfg.pe_ste), int(cfg.stop_grad_chunks),
                             L.ATLAS_BF16 if act_dtype == torch.bfloat16 else L.ATLAS_F32, cfg.precision)


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(dev):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _check_act(x, name, dtype, shape):
    if x.dtype != dtype or tuple(x.shape) != shape or not x.is_contiguous() or not x.is_cuda:
        raise ValueError(f"{name}: expected contiguous CUDA {dtype} {shape}, got {x.dtype} {tuple(x.shape)}")


class Workspace:
    """Grow-only scratch buffers reused across calls (the ABI itself never allocates).

    One buffer per (device, current stream): calls issued on different streams or
    devices never share scratch, and a buffer is only regrown by calls ordered on
    the stream that used it."""

    def __init__(self):
        self.bufs = {}

    def get(self, nbytes, device):
        if nbytes == 0:
            return None, 0
        key = (device, torch.cuda.current_stream(device).cuda_stream)
        buf = self.bufs.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = self.bufs[key] = torch.empty(nbytes, dtype=torch.uint8, device=device)
        return buf, buf.numel()


_WS = Workspace()


def saved_bytes(cfg, B, T, H, D, E, act_dtype=torch.bfloat16):
    lib = L.load()
    p = _params(cfg, B, T, H, D, E, act_dtype)
    n = lib.atlas_scan_saved_bytes(ctypes.byref(p))
    if n == 0:
        L.check(L.ATLAS_ERR_INVALID_ARGUMENT if lib.atlas_last_error_string() else L.ATLAS_OK)
    return n


def scan_forward(q, k, v, alpha, eta, theta, gamma=None, state=None, cfg=ScanConfig(), need_saved=True,
                 workspace=None):
    """Forward scan.  q,k,v: (B,T,H,D) float32 or bf16; gates (B,T,H) float32;
    state: (W1 (B,H,D,E), W2 (B,H,E,D), S1, S2) float32 or None for the LM init.
    Returns (y, (W1, W2, S1, S2), saved)."""
    lib = L.load()
    B, T, H, D = q.shape
    dev = q.device
    E = state[0].shape[-1] if state is not None else 4 * D
    return _forward(lib, q, k, v, alpha, eta, theta, gamma, state, cfg, need_saved, workspace, B, T, H, D, E,
                    dev)


def _forward(lib, q, k, v, alpha, eta, theta, gamma, state, cfg, need_saved, workspace, B, T, H, D, E, dev):
    for n, x in (("k", k), ("v", v)):
        _check_act(x, n, q.dtype, (B, T, H, D))
    for n, x in (("alpha", alpha), ("eta", eta), ("theta", theta), ("gamma", gamma)):
        if x is not None:
            _check_act(x, n, torch.float32, (B, T, H))
    p = _params(cfg, B, T, H, D, E, q.dtype)
    y = torch.empty_like(q)
    out = (torch.empty(B, H, D, E, device=dev), torch.empty(B, H, E, D, device=dev),
           torch.empty(B, H, D, E, device=dev), torch.empty(B, H, E, D, device=dev))
    nsave = lib.atlas_scan_saved_bytes(ctypes.byref(p)) if need_saved else 0
    if need_saved and nsave == 0:
        raise L.AtlasError(L.ATLAS_ERR_INVALID_ARGUMENT, lib.atlas_last_error_string().decode())
    saved = torch.empty(nsave, dtype=torch.uint8, device=dev) if need_saved else None
    ws, wsb = (workspace or _WS).get(lib.atlas_scan_workspace_bytes(ctypes.byref(p)), dev)
    st = [None] * 4 if state is None else [s.contiguous() for s in state]
    L.check(lib.atlas_scan_fwd(ctypes.byref(p), _ptr(q), _ptr(k), _ptr(v), _ptr(alpha), _ptr(eta), _ptr(theta),
                               _ptr(gamma), *[_ptr(s) for s in st], _ptr(y), *[_ptr(o) for o in out],
                               _ptr(saved), _ptr(ws), wsb, _stream(dev)))
    return y, out, saved


def scan_backward(q, k, v, alpha, eta, theta, gamma, saved, dy, dstate=None, cfg=ScanConfig(), E=None,
                  workspace=None):
    """VJP of ``scan_forward``.  Returns (dq, dk, dv, dalpha, deta, dtheta, dgamma, dstate_in)."""
    lib = L.load()
    B, T, H, D = q.shape
    dev = q.device
    E = E or 4 * D
    p = _params(cfg, B, T, H, D, E, q.dtype)
    _check_act(dy, "dy", q.dtype, (B, T, H, D))
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    g = [torch.empty(B, T, H, device=dev) for _ in range(4)]
    dst = (torch.empty(B, H, D, E, device=dev), torch.empty(B, H, E, D, device=dev),
           torch.empty(B, H, D, E, device=dev), torch.empty(B, H, E, D, device=dev))
    dso = [None] * 4 if dstate is None else [None if s is None else s.contiguous() for s in dstate]
    ws, wsb = (workspace or _WS).get(lib.atlas_scan_workspace_bytes(ctypes.byref(p)), dev)
    L.check(lib.atlas_scan_bwd(ctypes.byref(p), _ptr(q), _ptr(k), _ptr(v), _ptr(alpha), _ptr(eta), _ptr(theta),
                               _ptr(gamma), _ptr(saved), _ptr(dy), *[_ptr(s) for s in dso], _ptr(dq), _ptr(dk),
                               _ptr(dv), *[_ptr(x) for x in g], *[_ptr(s) for s in dst], _ptr(ws), wsb,
                               _stream(dev)))
    if gamma is None:
        g[3] = None
    return dq, dk, dv, g[0], g[1], g[2], g[3], dst


def linear_scan_forward(q, k, v, alpha, eta, theta, gamma=None, state=None, cfg=ScanConfig(), workspace=None):
    """Linear-memory scan (memory_layer.py:468-494), forward: q,k,v (B,T,H,D); gates
    (B,T,H) float32; state (M, S) each (B,H,D,D) float32 or None (zeros).
    Returns (y, (M, S)).  ATLAS_PREC_EXACT runs the float64 path (the one the backward
    uses); other precisions run the batched tensor-path forward."""
    lib = L.load()
    B, T, H, D = q.shape
    dev = q.device
    for n, x in (("k", k), ("v", v)):
        _check_act(x, n, q.dtype, (B, T, H, D))
    for n, x in (("alpha", alpha), ("eta", eta), ("theta", theta), ("gamma", gamma)):
        if x is not None:
            _check_act(x, n, torch.float32, (B, T, H))
    p = _params(cfg, B, T, H, D, D, q.dtype)
    y = torch.empty_like(q)
    out = (torch.empty(B, H, D, D, device=dev), torch.empty(B, H, D, D, device=dev))
    need = lib.atlas_linear_scan_workspace_bytes(ctypes.byref(p))
    if need == 0:
        raise L.AtlasError(L.ATLAS_ERR_UNSUPPORTED, lib.atlas_last_error_string().decode())
    ws, wsb = (workspace or _WS).get(need, dev)
    st = [None, None] if state is None else [s.contiguous() for s in state]
    L.check(lib.atlas_linear_scan_fwd(ctypes.byref(p), _ptr(q), _ptr(k), _ptr(v), _ptr(alpha), _ptr(eta),
                                      _ptr(theta), _ptr(gamma), _ptr(st[0]), _ptr(st[1]), _ptr(y),
                                      _ptr(out[0]), _ptr(out[1]), _ptr(ws), wsb, _stream(dev)))
    return y, out


def linear_scan_backward(q, k, v, alpha, eta, theta, gamma, state, dy, dstate=None, cfg=ScanConfig(),
                         workspace=None):
    """VJP of ``linear_scan_forward`` on the float64 path (cfg.precision must be
    ATLAS_PREC_EXACT).  Returns (dq, dk, dv, dalpha, deta, dtheta, dgamma, (dM, dS))."""
    lib = L.load()
    B, T, H, D = q.shape
    dev = q.device
    p = _params(cfg, B, T, H, D, D, q.dtype)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    g = [torch.empty(B, T, H, device=dev) for _ in range(4)]
    dst = (torch.empty(B, H, D, D, device=dev), torch.empty(B, H, D, D, device=dev))
    st = [None, None] if state is None else [s.contiguous() for s in state]
    dso = [None, None] if dstate is None else [None if s is None else s.contiguous() for s in dstate]
    need = lib.atlas_linear_scan_workspace_bytes(ctypes.byref(p))
    if need == 0:
        raise L.AtlasError(L.ATLAS_ERR_UNSUPPORTED, lib.atlas_last_error_string().decode())
    ws, wsb = (workspace or _WS).get(need, dev)
    L.check(lib.atlas_linear_scan_bwd(ctypes.byref(p), _ptr(q), _ptr(k), _ptr(v), _ptr(alpha), _ptr(eta),
                                      _ptr(theta), _ptr(gamma), _ptr(st[0]), _ptr(st[1]), _ptr(dy.contiguous()),
                                      _ptr(dso[0]), _ptr(dso[1]), _ptr(dq), _ptr(dk), _ptr(dv),
                                      *[_ptr(x) for x in g], _ptr(dst[0]), _ptr(dst[1]), _ptr(ws), wsb,
                                      _stream(dev)))
    if gamma is None:
        g[3] = None
    return dq, dk, dv, g[0], g[1], g[2], g[3], dst


def device_status():
    """Reads and clears the device status word (after a synchronize)."""
    code = L.load().atlas_scan_status()
    L.check(code)


def polar_express(X, steps=5, eps_in_sqrt=1e-12, precision=L.ATLAS_PREC_EXACT):
    """Batched Polar Express of a (..., rows, cols) float32 CUDA tensor."""
    lib = L.load()
    X = X.contiguous().float()
    rows, cols = X.shape[-2:]
    batch = X.numel() // (rows * cols)
    Y = torch.empty_like(X)
    ws, wsb = _WS.get(lib.atlas_polar_express_workspace_bytes(batch, rows, cols, steps, precision), X.device)
    L.check(lib.atlas_polar_express_batched(_ptr(X), _ptr(Y), batch, rows, cols, steps, eps_in_sqrt, precision,
                                            _ptr(ws), wsb, _stream(X.device)))
    return Y


class AtlasScan(torch.autograd.Function):
    """Autograd pairing of the forward and backward kernels (the analogue of the
    reference's jax.custom_vjp, fused_chunk.py:321-379)."""

    @staticmethod
    def forward(ctx, cfg, q, k, v, alpha, eta, theta, gamma, W1, W2, S1, S2):
        state = None if W1 is None else (W1, W2, S1, S2)
        E = W1.shape[-1] if W1 is not None else 4 * q.shape[-1]
        y, out, saved = _forward(L.load(), q, k, v, alpha, eta, theta, gamma, state, cfg, True, None,
                                 *q.shape, E, q.device)
        ctx.cfg, ctx.E = cfg, E
        ctx.save_for_backward(q, k, v, alpha, eta, theta, gamma, saved)
        ctx.has_state = state is not None
        return (y,) + tuple(out)

    @staticmethod
    def backward(ctx, dy, dW1, dW2, dS1, dS2):
        q, k, v, alpha, eta, theta, gamma, saved = ctx.saved_tensors
        dq, dk, dv, da, de, dt, dg, dst = scan_backward(q, k, v, alpha, eta, theta, gamma, saved,
                                                        dy.contiguous(), (dW1, dW2, dS1, dS2), ctx.cfg, ctx.E)
        if not ctx.has_state:
            dst = (None,) * 4
        return (None, dq, dk, dv, da, de, dt, dg) + tuple(dst)


def atlas_scan(q, k, v, alpha, eta, theta, gamma=None, state=None, cfg=ScanConfig()):
    """Differentiable scan: returns (y, (W1, W2, S1, S2))."""
    st = (None,) * 4 if state is None else tuple(state)
    out = AtlasScan.apply(cfg, q, k, v, alpha, eta, theta, gamma, *st)
    return out[0], tuple(out[1:])
