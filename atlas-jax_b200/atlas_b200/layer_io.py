"""Fused prologue / epilogue of the memory layer (include/atlas_layer.h).

``prologue`` replaces the elementwise half of atlas_jax/memory_layer.py:606-633
(ShortConv, rms_norm, polynomial features, sigmoid gates) and ``retrieve_gate``
replaces 720-722.  Both are autograd Functions over the C ABI; the projections
around them are plain GEMMs (torch.matmul, i.e. cuBLAS).
"""

import ctypes
from dataclasses import dataclass

import torch

from . import _lib as L
from .scan import _ptr, _stream


class AtlasLayerParams(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "abi_version", "B", "T", "H", "D", "conv_kernel", "poly_degree", "has_gamma", "has_retrieve",
        "act_dtype", "proj_stride")] + [("max_lr", ctypes.c_float)]


_P = ctypes.c_void_p
_bound = None


def _lib():
    global _bound
    lib = L.load()
    if _bound is None:
        pp = ctypes.POINTER(AtlasLayerParams)
        lib.atlas_layer_prologue_workspace_bytes.restype = ctypes.c_size_t
        lib.atlas_layer_prologue_workspace_bytes.argtypes = [pp]
        lib.atlas_layer_prologue_fwd.restype = ctypes.c_int
        lib.atlas_layer_prologue_fwd.argtypes = [pp] + [_P] * 5 + [_P] * 3 + [_P] * 5 + [_P]
        lib.atlas_layer_prologue_bwd.restype = ctypes.c_int
        lib.atlas_layer_prologue_bwd.argtypes = ([pp] + [_P] * 5 + [_P] * 3 + [_P] * 5 + [_P] * 5 +
                                                 [_P, ctypes.c_size_t, _P])
        lib.atlas_layer_retrieve_fwd.restype = ctypes.c_int
        lib.atlas_layer_retrieve_fwd.argtypes = [pp, _P, _P, _P, _P]
        lib.atlas_layer_retrieve_bwd.restype = ctypes.c_int
        lib.atlas_layer_retrieve_bwd.argtypes = [pp, _P, _P, _P, _P, _P, _P]
        _bound = True
    return lib


@dataclass(frozen=True)
class LayerGeometry:
    B: int
    T: int
    H: int
    D: int
    conv_kernel: int = 4
    poly_degree: int = 2
    has_gamma: bool = True
    has_retrieve: bool = True
    max_lr: float = 0.1
    pad_rows: bool = True  # proj rows padded to a multiple of 8 elements (16-byte lanes)

    @property
    def n_gates(self):
        return 3 + int(self.has_gamma) + int(self.has_retrieve)

    @property
    def n_proj(self):
        """Columns of the concatenated projection: q, k, v (H*D each) then the gates (H each)."""
        return 3 * self.H * self.D + self.n_gates * self.H

    @property
    def proj_stride(self):
        """Row stride of proj / dproj: n_proj rounded up to 8 (padding columns are zero)."""
        return (self.n_proj + 7) // 8 * 8 if self.pad_rows else self.n_proj

    def params(self, dtype):
        return AtlasLayerParams(L.ATLAS_ABI_VERSION, self.B, self.T, self.H, self.D, self.conv_kernel,
                                self.poly_degree, int(self.has_gamma), int(self.has_retrieve),
                                L.ATLAS_BF16 if dtype == torch.bfloat16 else L.ATLAS_F32, self.proj_stride,
                                self.max_lr)


def _need(x, dtype, shape, name):
    if x.dtype != dtype or tuple(x.shape) != tuple(shape) or not x.is_contiguous() or not x.is_cuda:
        raise ValueError(f"{name}: expected contiguous CUDA {dtype} {tuple(shape)}, got {x.dtype} {tuple(x.shape)}")


def prologue_forward(geo, proj, conv_w, conv_b, poly, gate_bias):
    """proj (B*T, proj_stride) act dtype -> q, k, v (B,T,H,D) act dtype and the gates (B,T,H) float32
    [alpha, eta, theta, gamma or None, retrieve or None]."""
    lib = _lib()
    B, T, H, D = geo.B, geo.T, geo.H, geo.D
    dt, dev = proj.dtype, proj.device
    _need(proj, dt, (B * T, geo.proj_stride), "proj")
    _need(conv_w, torch.float32, (3, geo.conv_kernel, H * D), "conv_w")
    _need(conv_b, torch.float32, (3, H * D), "conv_b")
    _need(gate_bias, torch.float32, (geo.n_gates - int(geo.has_retrieve), H), "gate_bias")
    p = geo.params(dt)
    q, k, v = (torch.empty(B, T, H, D, dtype=dt, device=dev) for _ in range(3))
    g = [torch.empty(B, T, H, device=dev) for _ in range(3)]
    g.append(torch.empty(B, T, H, device=dev) if geo.has_gamma else None)
    g.append(torch.empty(B, T, H, device=dev) if geo.has_retrieve else None)
    L.check(lib.atlas_layer_prologue_fwd(ctypes.byref(p), _ptr(proj), _ptr(conv_w), _ptr(conv_b), _ptr(poly),
                                         _ptr(gate_bias), _ptr(q), _ptr(k), _ptr(v), *[_ptr(x) for x in g],
                                         _stream(dev)))
    return q, k, v, g


def prologue_backward(geo, proj, conv_w, conv_b, poly, gate_bias, dq, dk, dv, dgates):
    """VJP of prologue_forward: returns dproj (act dtype), dconv_w, dconv_b, dpoly, dgate_bias."""
    lib = _lib()
    dt, dev = proj.dtype, proj.device
    p = geo.params(dt)
    dproj = torch.empty_like(proj)
    dcw, dcb = torch.empty_like(conv_w), torch.empty_like(conv_b)
    dpoly = torch.empty_like(poly) if poly is not None else None
    dgb = torch.empty_like(gate_bias)
    ws = torch.empty(lib.atlas_layer_prologue_workspace_bytes(ctypes.byref(p)), dtype=torch.uint8, device=dev)
    c = lambda x: None if x is None else x.contiguous()  # noqa: E731
    L.check(lib.atlas_layer_prologue_bwd(ctypes.byref(p), _ptr(proj), _ptr(conv_w), _ptr(conv_b), _ptr(poly),
                                         _ptr(gate_bias), _ptr(c(dq)), _ptr(c(dk)), _ptr(c(dv)),
                                         *[_ptr(c(x)) for x in dgates], _ptr(dproj), _ptr(dcw), _ptr(dcb),
                                         _ptr(dpoly), _ptr(dgb), _ptr(ws), ws.numel(), _stream(dev)))
    return dproj, dcw, dcb, dpoly, dgb


class Prologue(torch.autograd.Function):
    @staticmethod
    def forward(ctx, geo, proj, conv_w, conv_b, poly, gate_bias):
        q, k, v, g = prologue_forward(geo, proj, conv_w, conv_b, poly, gate_bias)
        ctx.geo = geo
        ctx.save_for_backward(proj, conv_w, conv_b, poly, gate_bias)
        return (q, k, v) + tuple(g)

    @staticmethod
    def backward(ctx, dq, dk, dv, da, de, dt, dg, dr):
        proj, conv_w, conv_b, poly, gate_bias = ctx.saved_tensors
        dproj, dcw, dcb, dpoly, dgb = prologue_backward(ctx.geo, proj, conv_w, conv_b, poly, gate_bias, dq, dk, dv,
                                                        (da, de, dt, dg, dr))
        return None, dproj, dcw, dcb, dpoly, dgb


def prologue(geo, proj, conv_w, conv_b, poly, gate_bias):
    """Differentiable fused prologue: (q, k, v, alpha, eta, theta, gamma, retrieve)."""
    return Prologue.apply(geo, proj, conv_w, conv_b, poly, gate_bias)


class RetrieveGate(torch.autograd.Function):
    @staticmethod
    def forward(ctx, geo, y, r):
        lib = _lib()
        p = geo.params(y.dtype)
        _need(y, y.dtype, (geo.B, geo.T, geo.H, geo.D), "y")
        _need(r, torch.float32, (geo.B, geo.T, geo.H), "retrieve")
        yg = torch.empty_like(y)
        L.check(lib.atlas_layer_retrieve_fwd(ctypes.byref(p), _ptr(y), _ptr(r), _ptr(yg), _stream(y.device)))
        ctx.geo = geo
        ctx.save_for_backward(y, r)
        return yg

    @staticmethod
    def backward(ctx, dyg):
        y, r = ctx.saved_tensors
        lib = _lib()
        p = ctx.geo.params(y.dtype)
        dyg = dyg.to(y.dtype).contiguous()
        dy, dr = torch.empty_like(y), torch.empty_like(r)
        L.check(lib.atlas_layer_retrieve_bwd(ctypes.byref(p), _ptr(y), _ptr(r), _ptr(dyg), _ptr(dy), _ptr(dr),
                                             _stream(y.device)))
        return None, dy, dr


def retrieve_gate(geo, y, r):
    """y * r[..., None] (memory_layer.py:720-722), differentiable."""
    return RetrieveGate.apply(geo, y, r)
