"""atlas_jax/kernels/b200_scan.py -- the reference-side binding of libatlas_scan.so.

UNTESTED HERE: this image and the GPU box have no JAX.  The file is written for the
reference's pinned jax/jaxlib 0.9.2 and is meant to be copied into
rkstgr/atlas-jax as ``atlas_jax/kernels/b200_scan.py``.  The C entry points it binds
(atlas_xla_fwd / atlas_xla_bwd, include/atlas_scan.h) are exercised on the B200 by
this repository's tests through the same buffer order (tests/test_gpu_xla.py).

It replaces the custom-VJP pair ``fused_chunk_scan`` (atlas_jax/kernels/fused_chunk.py:
321-379), called at memory_layer.py:535-541, with the whole scan of
``AtlasMemoryLayer.__call__`` (memory_layer.py:635-718): initial state, padding,
chunking and both directions run inside the library.

    y, state = atlas_scan(q, k, v, alpha, eta, theta, gamma, W1, W2, S_W1, S_W2,
                          chunk=64, omega=16, ns_steps=5, pe_ste=False,
                          stop_grad_chunks=False)

q, k, v: (B, T, H, D) float32 or bfloat16; gates (B, T, H) float32, already
activated; state float32 in the reference's layout (W1, S_W1 (B,H,D,E); W2, S_W2
(B,H,E,D)).  gamma is an array: pass ones when the layer has no gamma gate
(omega_window <= 1), which the window-1 aggregation never reads.
"""
import ctypes
import functools
import os

import jax
import jax.numpy as jnp
from jax.extend import core as jcore
from jax.interpreters import mlir
from jax._src.interpreters import mlir as _mlir

_LIB = ctypes.CDLL(os.environ.get("ATLAS_LIB_PATH", "libatlas_scan.so"))
_ABI_VERSION = 1
_F32, _BF16 = 0, 1
_PREC_TENSOR = 1


class _Params(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "abi_version", "B", "T", "H", "D", "E", "chunk", "omega", "ns_steps", "pe_ste",
        "stop_grad_chunks", "act_dtype", "precision")]


_LIB.atlas_scan_saved_bytes.restype = ctypes.c_size_t
_LIB.atlas_scan_workspace_bytes.restype = ctypes.c_size_t
_LIB.atlas_last_error_string.restype = ctypes.c_char_p
for _name in ("atlas_xla_fwd", "atlas_xla_bwd"):
    jax.ffi.register_ffi_target(_name, jax.ffi.pycapsule(getattr(_LIB, _name)), platform="CUDA",
                                api_version=0)


def _params(q, E, chunk, omega, ns_steps, pe_ste, stop_grad_chunks):
    B, T, H, D = q.shape
    act = _BF16 if q.dtype == jnp.bfloat16 else _F32
    p = _Params(_ABI_VERSION, B, T, H, D, E, chunk, omega, ns_steps, int(pe_ste), int(stop_grad_chunks), act,
                _PREC_TENSOR)
    saved = _LIB.atlas_scan_saved_bytes(ctypes.byref(p))
    ws = _LIB.atlas_scan_workspace_bytes(ctypes.byref(p))
    if saved == 0 or ws == 0:
        raise ValueError("atlas_scan: " + _LIB.atlas_last_error_string().decode())
    return bytes(p), saved, ws


def _lower(ctx, *operands, target, opaque):
    """Legacy status-returning custom call (api_version 2): buffers are the operands
    followed by the results, `opaque` travels as backend_config."""
    return _mlir.custom_call(
        target, result_types=[mlir.aval_to_ir_type(a) for a in ctx.avals_out], operands=list(operands),
        backend_config=opaque, api_version=2, has_side_effect=False).results


# ---- forward primitive: 11 operands -> y, W1, W2, S1, S2, saved, workspace ----
_fwd_p = jcore.Primitive("atlas_b200_scan_fwd")
_fwd_p.multiple_results = True


@_fwd_p.def_abstract_eval
def _fwd_abstract(q, k, v, a, e, t, g, W1, W2, S1, S2, *, opaque, saved, ws):
    f32 = jnp.float32
    return (jax.core.ShapedArray(q.shape, q.dtype), jax.core.ShapedArray(W1.shape, f32),
            jax.core.ShapedArray(W2.shape, f32), jax.core.ShapedArray(S1.shape, f32),
            jax.core.ShapedArray(S2.shape, f32), jax.core.ShapedArray((saved,), jnp.uint8),
            jax.core.ShapedArray((ws,), jnp.uint8))


mlir.register_lowering(_fwd_p, lambda ctx, *xs, opaque, saved, ws: _lower(ctx, *xs, target="atlas_xla_fwd",
                                                                           opaque=opaque), platform="cuda")

# ---- backward primitive: 13 operands -> dq, dk, dv, 4 gate grads, 4 state grads, workspace ----
_bwd_p = jcore.Primitive("atlas_b200_scan_bwd")
_bwd_p.multiple_results = True


@_bwd_p.def_abstract_eval
def _bwd_abstract(q, k, v, a, e, t, g, saved, dy, dW1, dW2, dS1, dS2, *, opaque, ws):
    f32 = jnp.float32
    return (jax.core.ShapedArray(q.shape, q.dtype),) * 3 + (jax.core.ShapedArray(a.shape, f32),) * 4 + \
        tuple(jax.core.ShapedArray(x.shape, f32) for x in (dW1, dW2, dS1, dS2)) + \
        (jax.core.ShapedArray((ws,), jnp.uint8),)


mlir.register_lowering(_bwd_p, lambda ctx, *xs, opaque, ws: _lower(ctx, *xs, target="atlas_xla_bwd",
                                                                    opaque=opaque), platform="cuda")


@functools.partial(jax.custom_vjp, nondiff_argnums=(11, 12, 13, 14, 15))
def atlas_scan(q, k, v, alpha, eta, theta, gamma, W1, W2, S1, S2,
               chunk=64, omega=16, ns_steps=5, pe_ste=False, stop_grad_chunks=False):
    out, _ = _scan_fwd(q, k, v, alpha, eta, theta, gamma, W1, W2, S1, S2,
                       chunk, omega, ns_steps, pe_ste, stop_grad_chunks)
    return out


def _scan_fwd(q, k, v, alpha, eta, theta, gamma, W1, W2, S1, S2, chunk, omega, ns_steps, pe_ste,
              stop_grad_chunks):
    opaque, saved_n, ws_n = _params(q, W1.shape[-1], chunk, omega, ns_steps, pe_ste, stop_grad_chunks)
    y, W1n, W2n, S1n, S2n, saved, _ = _fwd_p.bind(
        q, k, v, alpha, eta, theta, gamma, W1, W2, S1, S2, opaque=opaque, saved=saved_n, ws=ws_n)
    return (y, (W1n, W2n, S1n, S2n)), (q, k, v, alpha, eta, theta, gamma, saved)


def _scan_bwd(chunk, omega, ns_steps, pe_ste, stop_grad_chunks, res, ct):
    q, k, v, alpha, eta, theta, gamma, saved = res
    dy, (dW1, dW2, dS1, dS2) = ct  # custom_vjp materialises zero cotangents
    opaque, _, ws_n = _params(q, dW1.shape[-1], chunk, omega, ns_steps, pe_ste, stop_grad_chunks)
    f32 = lambda c: c.astype(jnp.float32)  # noqa: E731
    outs = _bwd_p.bind(q, k, v, alpha, eta, theta, gamma, saved, dy.astype(q.dtype),
                       f32(dW1), f32(dW2), f32(dS1), f32(dS2), opaque=opaque, ws=ws_n)
    dq, dk, dv, da, de, dt, dg, dW1i, dW2i, dS1i, dS2i, _ = outs
    return dq, dk, dv, da, de, dt, dg, dW1i, dW2i, dS1i, dS2i


atlas_scan.defvjp(_scan_fwd, _scan_bwd)



# ---- Muon: batched Polar Express of stacked parameter gradients (optim.py:68-83) ----
import struct  # noqa: E402

_LIB.atlas_polar_express_workspace_bytes.restype = ctypes.c_size_t
_LIB.atlas_polar_express_workspace_bytes.argtypes = [ctypes.c_int64] + [ctypes.c_int32] * 4
jax.ffi.register_ffi_target("atlas_xla_polar_express", jax.ffi.pycapsule(_LIB.atlas_xla_polar_express),
                            platform="CUDA", api_version=0)
_pe_p = jcore.Primitive("atlas_b200_polar_express")
_pe_p.multiple_results = True


@_pe_p.def_abstract_eval
def _pe_abstract(X, *, opaque, ws):
    return jax.core.ShapedArray(X.shape, jnp.float32), jax.core.ShapedArray((ws,), jnp.uint8)


mlir.register_lowering(_pe_p, lambda ctx, X, opaque, ws: _lower(ctx, X, target="atlas_xla_polar_express",
                                                                opaque=opaque), platform="cuda")


def muon_polar_express(g, ns_steps=5, precision=_PREC_TENSOR):
    """Drop-in for optim.py:68-83 (no 1e-12 inside the square root; tall matrices as
    X^T X, wide as X X^T): PE of a (..., rows, cols) gradient, returned in g's dtype."""
    rows, cols = g.shape[-2:]
    batch = 1
    for n in g.shape[:-2]:
        batch *= n
    ws = _LIB.atlas_polar_express_workspace_bytes(batch, rows, cols, ns_steps, precision)
    opaque = struct.pack("<qiiiifi", batch, rows, cols, ns_steps, precision, 0.0, 0)
    X, _ = _pe_p.bind(g.astype(jnp.float32), opaque=opaque, ws=ws)
    return X.astype(g.dtype)
