"""GPU parity of the tensor-path batched Polar Express (atlas_polar_express_batched
with ATLAS_PREC_TENSOR: three batched tcgen05 GEMMs per Newton-Schulz step on split
fp16 operands), the dispatch target of Muon's orthogonalisation
(atlas_jax/optim.py:68-83) and of the memory layer's Polar Express
(memory_layer.py:43-71).

Reference: a float64 torch restatement of the same iteration on the GPU (test
infrastructure), and the float64 exact path on a small case.  Shapes follow the
170M model's Muon stacks (768 x 768, 4096 x 768, 768 x 2048, the 12 x 768 gate
projections) plus ragged sizes that exercise the masked tile edges.  Tolerance
2e-4 relative (Frobenius; measured on B200 3e-8 to 6.4e-5, against 3e-6 to 5e-6
for a float32 torch restatement): the split keeps about 22 significant bits per
operand, and Polar Express amplifies rounding in the small singular directions.
"""
import pytest
import torch

from oracle import atlas_oracle as O

pytestmark = pytest.mark.gpu
TOL = 2e-4


def _ref(X, steps, eps, dtype=torch.float64):
    X = X.to(dtype)
    tall = X.shape[-2] > X.shape[-1]
    if tall:
        X = X.transpose(-1, -2)
    n = torch.sqrt((X * X).sum(dim=(-2, -1), keepdim=True) + eps)
    X = X / (n * 1.01 + 1e-6)
    for a, b, c in O.POLAR_EXPRESS_COEFFS[:steps]:
        A = X @ X.transpose(-1, -2)
        X = a * X + (b * A + c * A @ A) @ X
    return X.transpose(-1, -2) if tall else X


def _rel(a, b):
    return float((a.double() - b).norm() / b.norm())


@pytest.mark.parametrize("shape,steps,eps", [
    ((2, 768, 768), 5, 0.0),
    ((2, 2048, 768), 5, 0.0),
    ((1, 768, 2048), 5, 1e-12),
    ((3, 12, 768), 5, 0.0),
    ((2, 130, 200), 5, 1e-12),
    ((1, 4096, 768), 5, 0.0),
    ((2, 256, 96), 2, 0.0),
    ((2, 256, 96), 0, 0.0),
    ((2, 264, 200), 5, 0.0),
    ((3, 136, 1000), 5, 1e-12),
    ((4, 512, 128), 5, 0.0),
    ((3, 64, 256), 5, 0.0),
    ((5, 256, 64), 5, 1e-12),
    ((5, 64, 200), 5, 0.0),
    ((2, 64, 64), 5, 0.0),
    ((3, 64, 256), 0, 0.0),
    # head_dim 128 on the 2-CTA cluster kernel: wide and tall, E = 256 / 512, no steps,
    # and more matrices than resident clusters
    ((3, 128, 512), 5, 1e-12),
    ((2, 128, 256), 5, 0.0),
    ((2, 256, 128), 3, 0.0),
    ((2, 128, 512), 0, 0.0),
    ((200, 512, 128), 5, 0.0),
    # 64 x 256 on the on-chip per-CTA kernel: more pairs than CTAs, an odd tail, wide
    ((301, 256, 64), 5, 0.0),
    ((4, 64, 256), 4, 1e-12),
])
def test_tensor_pe_matches_float64(shape, steps, eps):
    from atlas_b200 import polar_express, ATLAS_PREC_TENSOR, device_status
    g = torch.Generator(device="cuda").manual_seed(hash(shape) % 1000 + steps)
    X = torch.randn(*shape, device="cuda", generator=g)
    Y = polar_express(X, steps, eps, precision=ATLAS_PREC_TENSOR)
    torch.cuda.synchronize()
    device_status()
    ref = _ref(X, steps, eps)
    err = _rel(Y, ref)
    torch.backends.cuda.matmul.allow_tf32 = False
    err32 = _rel(_ref(X, steps, eps, torch.float32), ref)
    print(shape, steps, f"kernel {err:.2e}  float32 restatement {err32:.2e}")
    assert Y.shape == X.shape and bool(torch.isfinite(Y).all())
    assert err < TOL, err


def test_tensor_pe_agrees_with_exact_path():
    from atlas_b200 import polar_express, ATLAS_PREC_TENSOR, ATLAS_PREC_EXACT
    X = torch.randn(3, 96, 160, device="cuda", generator=torch.Generator(device="cuda").manual_seed(5))
    Yt = polar_express(X, 5, 1e-12, precision=ATLAS_PREC_TENSOR)
    Ye = polar_express(X, 5, 1e-12, precision=ATLAS_PREC_EXACT)
    torch.cuda.synchronize()
    assert _rel(Yt, Ye.double()) < TOL
