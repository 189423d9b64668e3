"""GPU check of the Muon dispatch (atlas_b200.optim, the replacement of
atlas_jax/optim.py:56-108 whose Polar Express step 68-83 runs on the batched tcgen05
kernel): one Muon step on each of the 170M model's stacked matrix parameters
(12 layers of 768x768 attention/memory projections, the 4096x768 GeGLU input and
768x2048 output projections, and the 12x768 per-head gate projections) is compared
with a float64 torch restatement of the reference's leaf update.  Tolerance 1e-3
relative (measured up to 5.4e-4 on the 4096 x 768 stack: the NorMuon rescaling and
the cautious-decay mask amplify the Polar Express error of 6e-5)."""
import math

import pytest
import torch

from oracle import atlas_oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-3


def _ref_update(grad, mom, sm, param, lr, momentum, beta2, wd, ns):
    """optim.py:56-108 in float64."""
    shape = grad.shape
    lr_scale = math.sqrt(max(1.0, shape[-2] / shape[-1]))
    new_m = mom * momentum + grad * (1 - momentum)
    g = grad * (1 - momentum) + new_m * momentum
    X = g
    X = X / (torch.sqrt((X * X).sum(dim=(-2, -1), keepdim=True)) * 1.01 + 1e-6)
    tall = shape[-2] > shape[-1]
    T = lambda M: M.transpose(-1, -2)  # noqa: E731
    for a, b, c in O.POLAR_EXPRESS_COEFFS[:ns]:
        A = T(X) @ X if tall else X @ T(X)
        Bm = b * A + c * (A @ A)
        X = a * X + (X @ Bm if tall else Bm @ X)
    g = X
    red = -1 if shape[-2] >= shape[-1] else -2
    n = shape[red]
    v_mean = (g * g).mean(dim=red, keepdim=True)
    v_norm = torch.sqrt(v_mean.sum(dim=(-2, -1), keepdim=True) * n)
    new_sm = sm * beta2 + v_mean * (1 - beta2)
    step = torch.rsqrt(torch.clamp(new_sm, min=1e-10))
    v_norm_new = torch.sqrt(((v_mean * n) * step * step).sum(dim=(-2, -1), keepdim=True))
    g = g * (step * (v_norm / torch.clamp(v_norm_new, min=1e-10)))
    mask = (g * param) >= 0
    return -(lr * lr_scale * g + lr * lr_scale * wd * param * mask), new_m, new_sm


@pytest.mark.parametrize("shape", [(12, 768, 768), (12, 4096, 768), (12, 768, 2048), (12, 12, 768)])
def test_muon_step_on_170m_stacks(shape):
    from atlas_b200.optim import muon_init, muon_leaf_update
    gen = torch.Generator(device="cuda").manual_seed(sum(shape))
    param = 0.02 * torch.randn(shape, device="cuda", generator=gen)
    st = muon_init(param)
    st.momentum.copy_(0.01 * torch.randn(shape, device="cuda", generator=gen))
    st.second_moment.uniform_(0.0, 1e-3, generator=gen)
    grad = 0.01 * torch.randn(shape, device="cuda", generator=gen)
    upd, new = muon_leaf_update(grad, st, param, learning_rate=0.02, momentum=0.95, beta2=0.9,
                                weight_decay=0.1, ns_steps=5)
    torch.cuda.synchronize()
    r_upd, r_m, r_sm = _ref_update(grad.double(), st.momentum.double(), st.second_moment.double(),
                                   param.double(), 0.02, 0.95, 0.9, 0.1, 5)
    err = float((upd.double() - r_upd).norm() / r_upd.norm())
    print(shape, "update rel err", err)
    assert err < TOL
    assert float((new.momentum.double() - r_m).norm() / r_m.norm()) < 1e-6
    assert float((new.second_moment.double() - r_sm).norm() / r_sm.norm()) < TOL
