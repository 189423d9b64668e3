"""CPU checks of the C ABI library: it loads, exports every declared symbol,
and rejects bad arguments before touching the GPU."""
import ctypes

import pytest

from atlas_b200 import _lib as L


def test_library_exports_every_header_function():
    lib = L.load()
    names = L.header_functions()
    assert "atlas_scan_fwd" in names and "atlas_scan_bwd" in names
    for n in names:
        assert hasattr(lib, n), n
    assert lib.atlas_abi_version() == L.ATLAS_ABI_VERSION
    import os
    inc = os.path.dirname(L.HEADER)
    for h in sorted(os.listdir(inc)):  # every header in include/
        for n in L.header_functions(os.path.join(inc, h)):
            assert hasattr(lib, n), (h, n)


def _p(**kw):
    base = dict(B=2, T=100, H=3, D=32, E=128, chunk=64, omega=8, ns_steps=5, pe_ste=0, stop_grad_chunks=0,
                act_dtype=L.ATLAS_F32, precision=L.ATLAS_PREC_EXACT)
    base.update(kw)
    return L.AtlasScanParams(L.ATLAS_ABI_VERSION, *[base[k] for k in (
        "B", "T", "H", "D", "E", "chunk", "omega", "ns_steps", "pe_ste", "stop_grad_chunks", "act_dtype",
        "precision")])


def test_sizes_and_validation():
    lib = L.load()
    p = _p()
    # exact path saves float64 carries: B*H*ceil(T/cs)*4*D*E*8
    assert lib.atlas_scan_saved_bytes(ctypes.byref(p)) == 2 * 3 * 2 * 4 * 32 * 128 * 8
    assert lib.atlas_scan_workspace_bytes(ctypes.byref(p)) > 0
    bad = _p(ns_steps=7)
    assert lib.atlas_scan_saved_bytes(ctypes.byref(bad)) == 0
    assert b"ns_steps" in lib.atlas_last_error_string()
    bad = _p()
    bad.abi_version = 99
    rc = lib.atlas_scan_fwd(ctypes.byref(bad), *([None] * 18), 0, None)
    assert rc == L.ATLAS_ERR_INVALID_ARGUMENT
    rc = lib.atlas_scan_fwd(ctypes.byref(p), *([None] * 18), 0, None)
    assert rc == L.ATLAS_ERR_INVALID_ARGUMENT and b"non-NULL" in lib.atlas_last_error_string()


def test_polar_express_rejects_empty():
    lib = L.load()
    assert lib.atlas_polar_express_batched(None, None, 0, 4, 4, 5, 1e-12, 0, None, 0, None) \
        == L.ATLAS_ERR_INVALID_ARGUMENT


def test_polar_express_precisions():
    lib = L.load()
    # tensor path: the TMA GEMMs (where the driver offers tensor-map encoding) keep three
    # wide and three D x D float32 buffers plus 64 partial sums per matrix; the
    # register-staged GEMMs two of each
    tma = 12 * ((3 * 4096 * 768 + 3 * 768 * 768) * 4 + 64 * 8)
    staged = 12 * (2 * 4096 * 768 + 2 * 768 * 768) * 4
    assert lib.atlas_polar_express_workspace_bytes(12, 4096, 768, 5, L.ATLAS_PREC_TENSOR) in (tma, staged)
    assert lib.atlas_polar_express_workspace_bytes(12, 768, 768, 5, L.ATLAS_PREC_EXACT) > 0
    # an unknown precision is refused before any device work (the pointers are never read)
    dummy = ctypes.c_void_p(16)
    rc = lib.atlas_polar_express_batched(dummy, dummy, 1, 8, 8, 5, 0.0, 7, dummy, 1 << 20, None)
    assert rc == L.ATLAS_ERR_INVALID_ARGUMENT and b"precision" in lib.atlas_last_error_string()
    # too small a workspace is refused as well
    rc = lib.atlas_polar_express_batched(dummy, dummy, 1, 8, 8, 5, 0.0, L.ATLAS_PREC_TENSOR, dummy, 16, None)
    assert rc == L.ATLAS_ERR_WORKSPACE


def test_xla_adapters_reject_bad_opaque_and_report():
    """The XLA custom-call adapters validate the packed params before any device work
    and leave the message in atlas_last_error_string (status pointer NULL: no XLA)."""
    lib = L.load()
    assert lib.atlas_xla_opaque_bytes() == ctypes.sizeof(L.AtlasScanParams)
    bufs = (ctypes.c_void_p * 25)()
    lib.atlas_xla_fwd(None, bufs, b"short", 5, None)
    assert b"opaque" in lib.atlas_last_error_string()
    bad = _p(ns_steps=9)
    lib.atlas_xla_bwd(None, bufs, ctypes.string_at(ctypes.byref(bad), ctypes.sizeof(bad)), ctypes.sizeof(bad), None)
    assert b"ns_steps" in lib.atlas_last_error_string()


def test_noalloc_clears_error_and_returns_param_code():
    """atlas_scan_fwd_noalloc reports check failures with their own code (an
    unsupported tensor-path shape is ATLAS_ERR_UNSUPPORTED) and starts every call
    with an empty message."""
    lib = L.load()
    p = _p(precision=L.ATLAS_PREC_TENSOR)  # D=32: valid, but not a tensor-path shape
    rc = lib.atlas_scan_fwd_noalloc(ctypes.byref(p), *([None] * 16), None)
    assert rc == L.ATLAS_ERR_UNSUPPORTED and b"tensor path" in lib.atlas_last_error_string()
    bad = _p(ns_steps=9)
    rc = lib.atlas_scan_fwd_noalloc(ctypes.byref(bad), *([None] * 16), None)
    assert rc == L.ATLAS_ERR_INVALID_ARGUMENT and b"ns_steps" in lib.atlas_last_error_string()


def test_xla_polar_express_opaque_layout():
    """The Muon adapter's opaque is {int64 batch; int32 rows, cols, ns_steps, precision;
    float eps; int32 pad}, packed as the JAX binding packs it."""
    import struct
    lib = L.load()
    assert lib.atlas_xla_pe_opaque_bytes() == struct.calcsize("<qiiiifi") == 32
    bufs = (ctypes.c_void_p * 3)()
    lib.atlas_xla_polar_express(None, bufs, b"x" * 8, 8, None)
    assert b"AtlasXlaPEOpaque" in lib.atlas_last_error_string()


def test_batched_forward_sizes_and_backward_refusal():
    """Shapes outside the fused kernels (here D=128, E=512, chunk 128) take the batched
    tensor forward: it sizes a workspace, and the backward refuses them with
    ATLAS_ERR_UNSUPPORTED before touching the GPU."""
    lib = L.load()
    p = _p(D=128, E=512, chunk=128, precision=L.ATLAS_PREC_TENSOR)
    assert lib.atlas_scan_workspace_bytes(ctypes.byref(p)) > 0
    assert lib.atlas_scan_saved_bytes(ctypes.byref(p)) > 0
    rc = lib.atlas_scan_bwd(ctypes.byref(p), *([None] * 25), 0, None)
    assert rc == L.ATLAS_ERR_UNSUPPORTED and b"backward" in lib.atlas_last_error_string()
    bad = _p(D=48, precision=L.ATLAS_PREC_TENSOR_BATCHED)
    assert lib.atlas_scan_workspace_bytes(ctypes.byref(bad)) == 0
    assert b"head_dim" in lib.atlas_last_error_string()


def test_fused_forward_chunk_128_sizes_and_backward_refusal():
    """D=64, E=256 with chunk 128 runs the fused forward (factor scratch for 128-token
    chunks, no backward workspace); the backward refuses it before touching the GPU, and
    the no-alloc forward (sized for chunks <= 64) refuses it too."""
    lib = L.load()
    p64 = _p(D=64, E=256, chunk=64, precision=L.ATLAS_PREC_TENSOR)
    p128 = _p(D=64, E=256, chunk=128, precision=L.ATLAS_PREC_TENSOR)
    ws128 = lib.atlas_scan_workspace_bytes(ctypes.byref(p128))
    assert 0 < ws128 < lib.atlas_scan_workspace_bytes(ctypes.byref(p64))  # forward-only: no backward scratch
    nch = -(-100 // 128)
    assert lib.atlas_scan_saved_bytes(ctypes.byref(p128)) == 2 * 3 * nch * 4 * 64 * 256 * 4
    rc = lib.atlas_scan_bwd(ctypes.byref(p128), *([None] * 25), 0, None)
    assert rc == L.ATLAS_ERR_UNSUPPORTED and b"chunk" in lib.atlas_last_error_string()
    rc = lib.atlas_scan_fwd_noalloc(ctypes.byref(p128), *([None] * 16), None)
    assert rc == L.ATLAS_ERR_UNSUPPORTED
    p256 = _p(D=64, E=256, chunk=256, precision=L.ATLAS_PREC_TENSOR)
    assert lib.atlas_scan_workspace_bytes(ctypes.byref(p256)) > 0  # the batched forward takes it


def test_forward_only_few_chains_workspace_covers_the_batched_forward():
    """A forward-only ATLAS_PREC_TENSOR call with few chains may run the batched forward,
    so the workspace it is told to allocate covers that path too."""
    lib = L.load()
    p = _p(B=1, T=300, H=4, D=64, E=256, chunk=64, precision=L.ATLAS_PREC_TENSOR)
    pb = _p(B=1, T=300, H=4, D=64, E=256, chunk=64, precision=L.ATLAS_PREC_TENSOR_BATCHED)
    assert lib.atlas_scan_workspace_bytes(ctypes.byref(p)) >= lib.atlas_scan_workspace_bytes(ctypes.byref(pb)) > 0


def test_linear_scan_checks():
    lib = L.load()
    p = _p(D=64, precision=L.ATLAS_PREC_TENSOR)
    assert lib.atlas_linear_scan_workspace_bytes(ctypes.byref(p)) > 0
    ex = _p(D=64, precision=L.ATLAS_PREC_EXACT)
    assert lib.atlas_linear_scan_workspace_bytes(ctypes.byref(ex)) > 0
    rc = lib.atlas_linear_scan_fwd(ctypes.byref(ex), *([None] * 12), None, 0, None)
    assert rc == L.ATLAS_ERR_INVALID_ARGUMENT
    rc = lib.atlas_linear_scan_bwd(ctypes.byref(p), *([None] * 21), None, 0, None)
    assert rc == L.ATLAS_ERR_UNSUPPORTED and b"EXACT" in lib.atlas_last_error_string()
    rc = lib.atlas_linear_scan_bwd(ctypes.byref(ex), *([None] * 21), None, 0, None)
    assert rc == L.ATLAS_ERR_INVALID_ARGUMENT


def test_layer_io_exports_sizes_and_validation():
    import os
    from atlas_b200.layer_io import LayerGeometry, _lib
    lib = _lib()
    for n in L.header_functions(os.path.join(os.path.dirname(L.HEADER), "atlas_layer.h")):
        assert hasattr(lib, n), n
    geo = LayerGeometry(2, 50, 3, 64)
    assert geo.n_proj == 3 * 3 * 64 + 5 * 3
    p = geo.params(None)
    assert lib.atlas_layer_prologue_workspace_bytes(ctypes.byref(p)) == 2 * 50 * 3 * 3 * 64 * 4
    rc = lib.atlas_layer_prologue_fwd(ctypes.byref(p), *([None] * 14))
    assert rc == L.ATLAS_ERR_INVALID_ARGUMENT and b"NULL" in lib.atlas_last_error_string()
    bad = LayerGeometry(2, 50, 3, 512).params(None)
    assert lib.atlas_layer_prologue_workspace_bytes(ctypes.byref(bad)) == 0
    assert b"head_dim" in lib.atlas_last_error_string()
    bad = LayerGeometry(2, 50, 3, 64, conv_kernel=9).params(None)
    assert lib.atlas_layer_retrieve_fwd(ctypes.byref(bad), None, None, None, None) == L.ATLAS_ERR_INVALID_ARGUMENT
    # a valid check clears the message left by the failure above
    assert lib.atlas_layer_prologue_workspace_bytes(ctypes.byref(p)) > 0
    assert lib.atlas_last_error_string() == b""


def test_layer_io_argument_counts_match_header():
    """The ctypes prototypes have as many arguments as the C declarations."""
    import os
    import re
    from atlas_b200.layer_io import _lib
    lib = _lib()
    txt = open(os.path.join(os.path.dirname(L.HEADER), "atlas_layer.h")).read()
    for name, args in re.findall(r"(atlas_layer_\w+)\(([^;]*)\);", txt):
        assert len(getattr(lib, name).argtypes) == args.count(",") + 1, name
