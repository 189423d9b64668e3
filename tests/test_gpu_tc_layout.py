"""GPU check of the tcgen05 operand layouts (core-matrix tiles, K- and MN-major
descriptors, M=64 / M=128 TMEM accumulators) the scan kernels are built on."""
import ctypes
import itertools

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from atlas_b200 import _lib as L
    lib = L.load()
    lib.atlas_selftest_tc_gemm.restype = ctypes.c_int
    lib.atlas_selftest_tc_gemm.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int32] * 5 + [ctypes.c_void_p]
    return lib


@pytest.mark.parametrize("M,N,K,amn,bmn", [c for c in itertools.product((64, 128), (16, 64, 256), (16, 64, 256),
                                                                         (0, 1), (0, 1))])
def test_tc_gemm_layouts(M, N, K, amn, bmn):
    lib = _lib()
    g = torch.Generator().manual_seed(M * 1000 + N * 10 + K + amn * 7 + bmn * 3)
    A = torch.randn(M, K, generator=g).cuda()
    B = torch.randn(K, N, generator=g).cuda()
    D = torch.full((M, N), float("nan"), device="cuda")
    assert lib.atlas_selftest_tc_gemm(A.data_ptr(), B.data_ptr(), D.data_ptr(), M, N, K, amn, bmn, None) == 0
    torch.cuda.synchronize()
    ref = A.bfloat16().double() @ B.bfloat16().double()
    err = (D.double() - ref).abs().max().item() / ref.abs().max().item()
    assert err < 1e-5, err
