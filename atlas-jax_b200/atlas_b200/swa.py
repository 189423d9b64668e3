"""Banded causal attention with RoPE for the MAG hybrid (include/atlas_swa.h):
the attention core of atlas_jax/model.py:77-135 as an autograd Function over the
tcgen05 kernels, and ``SlidingWindowAttention`` with the reference's call shape
(rms_norm, to_qkv and to_out stay plain ops/GEMMs)."""

import ctypes
import math

import torch
import torch.nn as nn

from . import _lib as L
from .scan import _ptr, _stream


class AtlasSwaParams(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("abi_version", "B", "T", "H", "D", "window", "rope")]


_P = ctypes.c_void_p
_bound = False


def _lib():
    global _bound
    lib = L.load()
    if not _bound:
        pp = ctypes.POINTER(AtlasSwaParams)
        lib.atlas_swa_fwd.restype = ctypes.c_int
        lib.atlas_swa_fwd.argtypes = [pp, _P, _P, _P, _P, _P, _P, ctypes.c_size_t, _P]
        lib.atlas_swa_workspace_bytes.restype = ctypes.c_size_t
        lib.atlas_swa_workspace_bytes.argtypes = [pp]
        lib.atlas_swa_bwd.restype = ctypes.c_int
        lib.atlas_swa_bwd.argtypes = [pp] + [_P] * 9 + [_P, ctypes.c_size_t, _P]
        _bound = True
    return lib


def _params(q, window, rope):
    B, T, H, D = q.shape
    return AtlasSwaParams(L.ATLAS_ABI_VERSION, B, T, H, D, window, int(rope))


def swa_forward(q, k, v, window, rope=True):
    """q, k (pre-RoPE), v: (B, T, H, 64) bf16 -> (o, lse)."""
    lib = _lib()
    for n, x in (("q", q), ("k", k), ("v", v)):
        if x.dtype != torch.bfloat16 or not x.is_cuda or not x.is_contiguous() or x.shape != q.shape:
            raise ValueError(f"{n}: expected contiguous CUDA bf16 {tuple(q.shape)}")
    B, T, H, D = q.shape
    p = _params(q, window, rope)
    o = torch.empty_like(q)
    lse = torch.empty(B, H, T, device=q.device)
    ws = torch.empty(lib.atlas_swa_workspace_bytes(ctypes.byref(p)), dtype=torch.uint8, device=q.device)
    L.check(lib.atlas_swa_fwd(ctypes.byref(p), _ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(lse), _ptr(ws), ws.numel(),
                              _stream(q.device)))
    return o, lse


def swa_backward(q, k, v, o, lse, do, window, rope=True):
    lib = _lib()
    p = _params(q, window, rope)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    ws = torch.empty(lib.atlas_swa_workspace_bytes(ctypes.byref(p)), dtype=torch.uint8, device=q.device)
    L.check(lib.atlas_swa_bwd(ctypes.byref(p), _ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(lse),
                              _ptr(do.contiguous()), _ptr(dq), _ptr(dk), _ptr(dv), _ptr(ws), ws.numel(),
                              _stream(q.device)))
    return dq, dk, dv


class SwaFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, window, rope):
        o, lse = swa_forward(q, k, v, window, rope)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.window, ctx.rope = window, rope
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        dq, dk, dv = swa_backward(q, k, v, o, lse, do.to(torch.bfloat16), ctx.window, ctx.rope)
        return dq, dk, dv, None, None


def sliding_window_attention(q, k, v, window, rope=True):
    """Differentiable banded attention: (B, T, H, 64) bf16 in and out."""
    return SwaFunction.apply(q, k, v, window, rope)


def _rms_norm(x):
    xf = x.float()
    return (xf * torch.rsqrt((xf * xf).mean(-1, keepdim=True) + 1e-6)).to(x.dtype)


class SlidingWindowAttention(nn.Module):
    """model.py:77-135: rms_norm -> to_qkv -> banded RoPE attention -> to_out."""

    def __init__(self, n_embd, n_head, dim_head, window_size):
        super().__init__()
        self.n_head, self.dim_head, self.window_size = n_head, dim_head, window_size
        self.to_qkv = nn.Linear(n_embd, 3 * n_head * dim_head, bias=False)
        self.to_out = nn.Linear(n_head * dim_head, n_embd, bias=False)

    def forward(self, x):
        B, T, C = x.shape
        H, D = self.n_head, self.dim_head
        qkv = self.to_qkv(_rms_norm(x)).to(torch.bfloat16)
        q, k, v = (t.reshape(B, T, H, D).contiguous() for t in qkv.split(H * D, dim=-1))
        o = sliding_window_attention(q, k, v, self.window_size)
        return self.to_out(o.reshape(B, T, H * D).to(x.dtype))


if __name__ == "__main__":
    # Profiling case: seeded bf16 q, k, v, dO of shape (1, 32768, 12, 64), window 1024,
    # forward + backward twice (python -m atlas_b200.swa from atlas-jax_b200/).
    g = torch.Generator(device="cuda")
    g.manual_seed(0)
    q, k, v, do = (torch.randn(1, 32768, 12, 64, device="cuda", generator=g).to(torch.bfloat16) for _ in range(4))
    for _ in range(2):
        o, lse = swa_forward(q, k, v, 1024)
        swa_backward(q, k, v, o, lse, do, 1024)
    torch.cuda.synchronize()
    print("ok")
