"""torch float64 restatement of the memory layer's prologue and retrieve gate
(atlas_jax/memory_layer.py:606-633, 720-722) on the concatenated projection, for
autograd checks of the fused kernels' VJPs (test infrastructure)."""
import numpy as np
import torch


def prologue(proj, B, T, H, D, conv_w, conv_b, poly, gate_bias, has_gamma, has_retrieve, max_lr):
    di = H * D
    P = proj.reshape(B, T, -1)
    K = conv_w.shape[-1]
    outs = []
    for i in range(3):
        x = P[..., i * di:(i + 1) * di].transpose(1, 2)
        x = torch.nn.functional.pad(x, (K - 1, 0))
        y = torch.nn.functional.conv1d(x, conv_w[i].unsqueeze(1), conv_b[i], groups=di)
        outs.append(y.transpose(1, 2).reshape(B, T, H, D))
    q, k, v = outs
    rms = lambda z: z * torch.rsqrt((z * z).mean(-1, keepdim=True) + 1e-6)  # noqa: E731

    def phi(z):
        out, zp = poly[0] * z, z
        for i in range(1, poly.shape[0]):
            zp = zp * z
            out = out + poly[i] * zp
        return out
    if poly is not None and poly.shape[0] > 0:
        q, k = phi(rms(q)), rms(phi(k))
    else:
        q, k = rms(q), rms(k)
    names = ["alpha", "eta", "theta"] + (["gamma"] if has_gamma else []) + (["retrieve"] if has_retrieve else [])
    g = {}
    for i, n in enumerate(names):
        z = P[..., 3 * di + i * H:3 * di + (i + 1) * H]
        if n != "retrieve":
            z = z + gate_bias[i]
        s = torch.sigmoid(z)
        g[n] = s * max_lr if n == "eta" else s
    return q, k, v, [g.get(n) for n in ("alpha", "eta", "theta", "gamma", "retrieve")]


def make_params(H, D, K, poly_degree, n_bias, seed=0):
    rng = np.random.default_rng(seed)
    conv_w = (rng.standard_normal((3, H * D, K)) * 0.3).astype(np.float32)
    conv_b = (rng.standard_normal((3, H * D)) * 0.1).astype(np.float32)
    poly = (1.0 + 0.3 * rng.standard_normal(poly_degree)).astype(np.float32) if poly_degree else None
    gate_bias = rng.standard_normal((n_bias, H)).astype(np.float32)
    return conv_w, conv_b, poly, gate_bias
