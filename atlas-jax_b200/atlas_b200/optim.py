"""Muon dispatch onto the batched Polar Express kernels.

Mirrors the Muon leaf update of the reference (atlas_jax/optim.py:56-108,
``_muon_leaf_update``) for torch CUDA tensors.  Its Polar Express step
(optim.py:68-83: Frobenius pre-normalisation without the 1e-12 inside the square
root, tall matrices as X^T X, wide as X X^T) runs in libatlas_scan.so through
``atlas_polar_express_batched``; a stacked parameter (L, rows, cols) is one batched
call.  The momentum, NorMuon and weight-decay arithmetic around it is elementwise
and stays in torch.
"""
import math
from dataclasses import dataclass

import torch

from . import _lib as L
from .scan import polar_express


def muon_polar_express(g, ns_steps=5, precision=L.ATLAS_PREC_TENSOR):
    """optim.py:68-83 for a (..., rows, cols) gradient: returns PE(g) in g's dtype.
    ATLAS_PREC_TENSOR runs the three tcgen05 GEMMs per step; ATLAS_PREC_EXACT runs
    float64 on CUDA cores (small matrices, checks)."""
    if g.dim() < 2:
        raise ValueError("Muon applies to matrices (..., rows, cols)")
    X = polar_express(g.float(), steps=ns_steps, eps_in_sqrt=0.0, precision=precision)
    return X.to(g.dtype)


@dataclass
class MuonState:
    momentum: torch.Tensor        # first moment (optim.py:37)
    second_moment: torch.Tensor   # NorMuon factored second moment (optim.py:38)


def muon_init(param):
    """optim.py:46-55."""
    shape = param.shape
    sm = (*shape[:-2], shape[-2], 1) if shape[-2] >= shape[-1] else (*shape[:-2], 1, shape[-1])
    return MuonState(torch.zeros_like(param), torch.zeros(sm, dtype=param.dtype, device=param.device))


def muon_leaf_update(grad, state, param, learning_rate, momentum=0.95, beta2=0.9, weight_decay=0.0, ns_steps=5,
                     precision=L.ATLAS_PREC_TENSOR):
    """One Muon step of one (possibly stacked) matrix parameter, optim.py:56-108.
    Returns (update, new_state)."""
    dtype, shape = grad.dtype, grad.shape
    lr_scale = math.sqrt(max(1.0, shape[-2] / shape[-1]))
    new_m = state.momentum * momentum + grad * (1 - momentum)            # Nesterov (61-63)
    g = grad * (1 - momentum) + new_m * momentum
    g = muon_polar_express(g, ns_steps, precision)                       # 65-84 on the kernel
    red = -1 if shape[-2] >= shape[-1] else -2                            # NorMuon (86-100)
    n = shape[red]
    gf = g.float()
    v_mean = (gf * gf).mean(dim=red, keepdim=True)
    v_norm = torch.sqrt(v_mean.sum(dim=(-2, -1), keepdim=True) * n)
    new_sm = state.second_moment * beta2 + v_mean.to(dtype) * (1 - beta2)
    step = torch.rsqrt(torch.clamp(new_sm, min=1e-10).float())
    v_norm_new = torch.sqrt(((v_mean * n) * step * step).sum(dim=(-2, -1), keepdim=True))
    g = g * (step * (v_norm / torch.clamp(v_norm_new, min=1e-10))).to(dtype)
    if param is not None and weight_decay > 0:                           # cautious decay (102-106)
        mask = (g * param) >= 0
        update = -(learning_rate * lr_scale * g + learning_rate * lr_scale * weight_decay * param * mask)
    else:
        update = -learning_rate * lr_scale * g
    return update, MuonState(new_m, new_sm)


if __name__ == "__main__":
    # Profiling case: a seeded float32 stack (default 12 x 768 x 2048, or "NxRxC" as the
    # first argument), five-step tensor-path Polar Express twice
    # (python -m atlas_b200.optim from atlas-jax_b200/).
    import sys
    shape = tuple(int(x) for x in (sys.argv[1] if len(sys.argv) > 1 else "12x768x2048").split("x"))
    gen = torch.Generator(device="cuda")
    gen.manual_seed(0)
    X = torch.randn(*shape, device="cuda", generator=gen)
    for _ in range(2):
        muon_polar_express(X, 5)
    torch.cuda.synchronize()
    print("ok")
