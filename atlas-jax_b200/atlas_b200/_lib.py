"""ctypes binding of libatlas_scan.so (include/atlas_scan.h).

The library is required: importing this module raises if it is missing, and
there is no CPU or PyTorch fallback for any entry point.
"""

import ctypes
import os
import re

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("ATLAS_LIB_PATH") or os.path.join(_HERE, "libatlas_scan.so")
HEADER = os.path.join(os.path.dirname(os.path.dirname(_HERE)), "include", "atlas_scan.h")

ATLAS_ABI_VERSION = 1
ATLAS_OK, ATLAS_ERR_INVALID_ARGUMENT, ATLAS_ERR_UNSUPPORTED, ATLAS_ERR_CUDA, ATLAS_ERR_DEVICE_TIMEOUT, \
    ATLAS_ERR_WORKSPACE = range(6)
ATLAS_F32, ATLAS_BF16 = 0, 1
ATLAS_PREC_EXACT, ATLAS_PREC_TENSOR, ATLAS_PREC_TENSOR_BATCHED = 0, 1, 2


class AtlasScanParams(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "abi_version", "B", "T", "H", "D", "E", "chunk", "omega", "ns_steps", "pe_ste",
        "stop_grad_chunks", "act_dtype", "precision")]


class AtlasError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"atlas error {code}: {msg}")
        self.code = code


_lib = None
_P = ctypes.c_void_p
_F = ctypes.c_void_p  # float* passed as raw addresses


def load():
    """Loads the library once; raises OSError if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise OSError(f"{LIB_PATH} not found: build it with `python atlas-jax_b200/build.py`")
    lib = ctypes.CDLL(LIB_PATH)
    pp = ctypes.POINTER(AtlasScanParams)
    lib.atlas_abi_version.restype = ctypes.c_int
    lib.atlas_last_error_string.restype = ctypes.c_char_p
    lib.atlas_scan_saved_bytes.restype = ctypes.c_size_t
    lib.atlas_scan_saved_bytes.argtypes = [pp]
    lib.atlas_scan_workspace_bytes.restype = ctypes.c_size_t
    lib.atlas_scan_workspace_bytes.argtypes = [pp]
    lib.atlas_scan_fwd.restype = ctypes.c_int
    lib.atlas_scan_fwd.argtypes = [pp] + [_P] * 3 + [_F] * 4 + [_F] * 4 + [_P] + [_F] * 4 + [_P, _P,
                                                                                                ctypes.c_size_t, _P]
    lib.atlas_scan_bwd.restype = ctypes.c_int
    lib.atlas_scan_bwd.argtypes = ([pp] + [_P] * 3 + [_F] * 4 + [_P, _P] + [_F] * 4 + [_P] * 3 + [_F] * 4
                                   + [_F] * 4 + [_P, ctypes.c_size_t, _P])
    lib.atlas_polar_express_batched.restype = ctypes.c_int
    lib.atlas_polar_express_batched.argtypes = [_F, _F, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                                ctypes.c_int32, ctypes.c_float, ctypes.c_int32, _P,
                                                ctypes.c_size_t, _P]
    lib.atlas_polar_express_workspace_bytes.restype = ctypes.c_size_t
    lib.atlas_polar_express_workspace_bytes.argtypes = [ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                                        ctypes.c_int32, ctypes.c_int32]
    lib.atlas_scan_status.restype = ctypes.c_int
    lib.atlas_debug_set_wait_hooks.restype = ctypes.c_int
    lib.atlas_debug_set_wait_hooks.argtypes = [ctypes.c_int32, ctypes.c_int32]
    lib.atlas_scan_fwd_noalloc.restype = ctypes.c_int
    lib.atlas_scan_fwd_noalloc.argtypes = [pp] + [_P] * 3 + [_F] * 4 + [_F] * 4 + [_P] + [_F] * 4 + [_P]
    lib.atlas_linear_scan_workspace_bytes.restype = ctypes.c_size_t
    lib.atlas_linear_scan_workspace_bytes.argtypes = [pp]
    lib.atlas_linear_scan_fwd.restype = ctypes.c_int
    lib.atlas_linear_scan_fwd.argtypes = [pp] + [_P] * 3 + [_F] * 4 + [_F] * 2 + [_P] + [_F] * 2 + [_P, ctypes.c_size_t,
                                                                                                  _P]
    lib.atlas_linear_scan_bwd.restype = ctypes.c_int
    lib.atlas_linear_scan_bwd.argtypes = [pp] + [_P] * 3 + [_F] * 4 + [_F] * 2 + [_P] + [_F] * 2 + [_P] * 3 + \
        [_F] * 4 + [_F] * 2 + [_P, ctypes.c_size_t, _P]
    lib.atlas_xla_opaque_bytes.restype = ctypes.c_size_t
    lib.atlas_xla_pe_opaque_bytes.restype = ctypes.c_size_t
    for n in ("atlas_xla_fwd", "atlas_xla_bwd", "atlas_xla_polar_express"):
        getattr(lib, n).restype = None
        getattr(lib, n).argtypes = [_P, ctypes.POINTER(ctypes.c_void_p), ctypes.c_char_p, ctypes.c_size_t, _P]
    if lib.atlas_abi_version() != ATLAS_ABI_VERSION:
        raise OSError(f"libatlas_scan ABI {lib.atlas_abi_version()} != {ATLAS_ABI_VERSION}")
    _lib = lib
    return lib


def check(code):
    if code != ATLAS_OK:
        raise AtlasError(code, load().atlas_last_error_string().decode())


def header_functions(header=HEADER):
    """Names of the functions a header in include/ declares."""
    txt = open(header).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\*?(atlas_\w+)\s*\(", txt, re.M)))
