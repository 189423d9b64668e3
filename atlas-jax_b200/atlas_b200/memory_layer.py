"""Host-side mirror of the reference's AtlasMemoryLayer (atlas_jax/memory_layer.py:336-727)
with its scan running on the B200 kernels.

Same constructor fields (AtlasConfig, atlas_jax/config.py:6-33) and the same call
signature, ``layer(x, memory_state=None) -> (y, DeepMemoryState)``.  The
projections, short convolutions, normalisation, gates, retrieve gate and output
projection (memory_layer.py:606-633, 720-725) stay ordinary torch ops around the
scan, exactly where the reference keeps them in XLA; the scan itself
(memory_layer.py:635-718) is one call to the C ABI through ``AtlasScan`` (forward
and backward kernels), with no PyTorch fallback.
"""

import math
from dataclasses import dataclass
from typing import NamedTuple, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from .scan import ScanConfig, atlas_scan
from . import _lib as L


@dataclass
class AtlasConfig:
    """The fields of atlas_jax/config.py:6-33 that the memory layer reads."""
    n_embd: int = 768
    n_head: int = 12
    dim_head: Optional[int] = None
    chunk_size: int = 64
    conv_kernel: int = 4
    ns_steps: int = 5
    omega_window: int = 16
    poly_degree: int = 2
    deep_memory: bool = True
    memory_expand: int = 4
    pe_ste: bool = False
    use_checkpoint: bool = True
    max_lr: float = 0.1
    stop_grad_chunks: bool = False


class DeepMemoryState(NamedTuple):
    """memory_layer.py:106-115: W1, S_W1 (B,H,D,E); W2, S_W2 (B,H,E,D)."""
    W1: torch.Tensor
    W2: torch.Tensor
    S_W1: torch.Tensor
    S_W2: torch.Tensor


def rms_norm(x):
    """memory_layer.py:211-216 (computed in float32)."""
    xf = x.float()
    return (xf * torch.rsqrt((xf * xf).mean(-1, keepdim=True) + 1e-6)).to(x.dtype)


class ShortConv(nn.Module):
    """Causal depthwise 1-D convolution, memory_layer.py:303-329."""

    def __init__(self, dim, kernel_size=4):
        super().__init__()
        self.kernel_size = kernel_size
        self.weight = nn.Parameter(torch.randn(dim, 1, kernel_size) * 0.02)
        self.bias = nn.Parameter(torch.zeros(dim))

    def forward(self, x):  # (B, T, C)
        xt = F.pad(x.transpose(1, 2), (self.kernel_size - 1, 0))
        y = F.conv1d(xt, self.weight.to(x.dtype), self.bias.to(x.dtype), groups=x.shape[-1])
        return y.transpose(1, 2)


class AtlasMemoryLayer(nn.Module):
    """Deep-memory Atlas layer (memory_layer.py:336-727), scan on the B200 kernels.

    ``precision`` selects the scan arithmetic: ATLAS_PREC_TENSOR (tcgen05, head_dim
    64 / memory hidden 256) or ATLAS_PREC_EXACT (float64 CUDA cores, any shape)."""

    def __init__(self, config: AtlasConfig, precision=L.ATLAS_PREC_TENSOR):
        super().__init__()
        if not config.deep_memory:
            raise NotImplementedError("only the deep (MLP) memory is on the B200 path")
        H = config.n_head
        D = config.dim_head if config.dim_head is not None else config.n_embd // H
        E = config.memory_expand * D
        C, di = config.n_embd, H * D
        self.config, self.n_head, self.head_dim, self.expand_dim = config, H, D, E
        self.c_q = nn.Linear(C, di, bias=False)
        self.c_k = nn.Linear(C, di, bias=False)
        self.c_v = nn.Linear(C, di, bias=False)
        self.c_proj = nn.Linear(di, C, bias=False)
        self.conv_q = ShortConv(di, config.conv_kernel)
        self.conv_k = ShortConv(di, config.conv_kernel)
        self.conv_v = ShortConv(di, config.conv_kernel)
        self.gate_alpha = nn.Linear(C, H)
        self.gate_eta = nn.Linear(C, H)
        self.gate_theta = nn.Linear(C, H)
        self.gate_gamma = nn.Linear(C, H) if config.omega_window > 1 else None
        self.poly_coeffs = nn.Parameter(torch.ones(config.poly_degree)) if config.poly_degree > 0 else None
        self.ln_gamma = nn.Parameter(torch.zeros(H, D))  # present in the reference, unused by its __call__
        b = math.sqrt(6.0 / (D + E))                      # Xavier-uniform, memory_layer.py:448-452
        self.W1_init = nn.Parameter(torch.empty(H, D, E).uniform_(-b, b))
        self.W2_init = nn.Parameter(torch.empty(H, E, D).uniform_(-b, b))
        self.retrieve_gate = nn.Linear(C, H, bias=False) if H > 1 else None
        self.scan_cfg = ScanConfig(chunk=config.chunk_size, omega=config.omega_window, ns_steps=config.ns_steps,
                                   pe_ste=config.pe_ste, stop_grad_chunks=config.stop_grad_chunks,
                                   precision=precision)

    def _poly(self, x):
        out = self.poly_coeffs[0] * x
        xp = x
        for i in range(1, self.config.poly_degree):
            xp = xp * x
            out = out + self.poly_coeffs[i] * xp
        return out

    def forward(self, x, memory_state=None):
        B, T, C = x.shape
        H, D, E = self.n_head, self.head_dim, self.expand_dim
        q = self.conv_q(self.c_q(x)).reshape(B, T, H, D)      # memory_layer.py:606-609
        k = self.conv_k(self.c_k(x)).reshape(B, T, H, D)
        v = self.conv_v(self.c_v(x)).reshape(B, T, H, D)
        if self.poly_coeffs is not None:                       # 611-618
            q = self._poly(rms_norm(q))
            k = rms_norm(self._poly(k))
        else:
            q, k = rms_norm(q), rms_norm(k)
        alpha = torch.sigmoid(self.gate_alpha(x)).float()     # 620-633, gates already activated
        eta = (torch.sigmoid(self.gate_eta(x)) * self.config.max_lr).float()
        theta = torch.sigmoid(self.gate_theta(x)).float()
        gamma = torch.sigmoid(self.gate_gamma(x)).float() if self.gate_gamma is not None else None
        if memory_state is None:                               # 635-643
            W1 = self.W1_init.float().unsqueeze(0).expand(B, H, D, E).contiguous()
            W2 = self.W2_init.float().unsqueeze(0).expand(B, H, E, D).contiguous()
            memory_state = DeepMemoryState(W1, W2, torch.zeros_like(W1), torch.zeros_like(W2))
        act = torch.bfloat16 if x.dtype == torch.bfloat16 else torch.float32
        y, st = atlas_scan(q.to(act).contiguous(), k.to(act).contiguous(), v.to(act).contiguous(),
                           alpha.contiguous(), eta.contiguous(), theta.contiguous(),
                           None if gamma is None else gamma.contiguous(),
                           tuple(s.float().contiguous() for s in memory_state), self.scan_cfg)
        y = y.to(x.dtype)
        if self.retrieve_gate is not None:                     # 720-722
            y = y * torch.sigmoid(self.retrieve_gate(x)).unsqueeze(-1)
        y = self.c_proj(y.reshape(B, T, H * D))                # 724-725
        return y, DeepMemoryState(*st)
