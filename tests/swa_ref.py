"""torch float64 restatement of SlidingWindowAttention's core (atlas_jax/model.py:49-75
RoPE, 117-133 scores / mask / softmax / values), dense T x T, for checking the
banded kernels (test infrastructure)."""
import torch


def rope(x):
    """x (B, T, H, D): halves rotated by position, inv_freq = 10000^(-2i/D) (model.py:54-75)."""
    B, T, H, D = x.shape
    inv = 1.0 / (10000.0 ** (torch.arange(0, D, 2, dtype=torch.float32) / D))
    fr = torch.outer(torch.arange(T, dtype=torch.float32), inv).to(x.dtype)
    cos, sin = fr.cos()[None, :, None, :], fr.sin()[None, :, None, :]
    x1, x2 = x[..., :D // 2], x[..., D // 2:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], -1)


def attention(q, k, v, window, use_rope=True):
    B, T, H, D = q.shape
    if use_rope:
        q, k = rope(q), rope(k)
    s = torch.einsum('bqhd,bkhd->bhqk', q, k) / D ** 0.5
    qp = torch.arange(T)[:, None]
    kp = torch.arange(T)[None, :]
    mask = (qp >= kp) & ((qp - kp) <= window)
    s = torch.where(mask, s, torch.full_like(s, -1e9))
    p = torch.softmax(s, -1)
    return torch.einsum('bhqk,bkhd->bqhd', p, v), torch.logsumexp(s, -1)
