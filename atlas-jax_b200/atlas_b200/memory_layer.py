"""Host-side mirror of the reference's AtlasMemoryLayer (atlas_jax/memory_layer.py:336-727)
with its scan running on the B200 kernels.

Same constructor fields (AtlasConfig, atlas_jax/config.py:6-33) and the same call
signature, ``layer(x, memory_state=None) -> (y, DeepMemoryState)``.  Per call:
one GEMM of x against every projection (q, k, v, the gates and the retrieve gate,
concatenated), the fused prologue kernel (short convolutions, rms_norm, polynomial
features, sigmoid gates; memory_layer.py:606-633), the scan (635-718) through
``AtlasScan``, the fused retrieve gate (720-722) and the c_proj GEMM (724-725).
Every non-GEMM step runs in libatlas_scan.so, forward and backward; there is no
PyTorch fallback.
"""

import math
from dataclasses import dataclass
from typing import NamedTuple, Optional

import torch
import torch.nn as nn

from .scan import ScanConfig, atlas_scan
from .layer_io import LayerGeometry, prologue, retrieve_gate
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


class ShortConv(nn.Module):
    """Parameters of a causal depthwise 1-D convolution (memory_layer.py:303-329); the
    convolution itself runs inside the fused prologue kernel."""

    def __init__(self, dim, kernel_size=4):
        super().__init__()
        self.kernel_size = kernel_size
        self.weight = nn.Parameter(torch.randn(dim, 1, kernel_size) * 0.02)
        self.bias = nn.Parameter(torch.zeros(dim))


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

    def geometry(self, B, T):
        cfg = self.config
        return LayerGeometry(B, T, self.n_head, self.head_dim, cfg.conv_kernel, cfg.poly_degree if
                             self.poly_coeffs is not None else 0, self.gate_gamma is not None,
                             self.retrieve_gate is not None, cfg.max_lr)

    def _fused_weights(self):
        """The projections as one GEMM operand and the prologue's parameter stacks."""
        lin = [self.c_q, self.c_k, self.c_v, self.gate_alpha, self.gate_eta, self.gate_theta]
        gates = [self.gate_alpha, self.gate_eta, self.gate_theta]
        if self.gate_gamma is not None:
            lin.append(self.gate_gamma)
            gates.append(self.gate_gamma)
        if self.retrieve_gate is not None:
            lin.append(self.retrieve_gate)
        W = torch.cat([m.weight for m in lin], 0)
        pad = self.geometry(1, 1).proj_stride - W.shape[0]  # zero rows: 16-byte aligned projection rows
        if pad:
            W = torch.cat([W, W.new_zeros(pad, W.shape[1])], 0)
        conv_w = torch.stack([c.weight[:, 0, :].t() for c in (self.conv_q, self.conv_k, self.conv_v)]).float()  # (3, K, di)
        conv_b = torch.stack([c.bias for c in (self.conv_q, self.conv_k, self.conv_v)]).float()
        gate_b = torch.stack([m.bias for m in gates]).float()
        poly = self.poly_coeffs.float() if self.poly_coeffs is not None else None
        return W, conv_w.contiguous(), conv_b.contiguous(), gate_b.contiguous(), poly

    def forward(self, x, memory_state=None):
        B, T, C = x.shape
        H, D, E = self.n_head, self.head_dim, self.expand_dim
        geo = self.geometry(B, T)
        act = torch.bfloat16 if x.dtype == torch.bfloat16 else torch.float32
        W, conv_w, conv_b, gate_b, poly = self._fused_weights()
        # memory_layer.py:606-633: one GEMM for every projection, then the fused prologue
        proj = (x.reshape(B * T, C).to(act) @ W.to(act).T).contiguous()
        q, k, v, alpha, eta, theta, gamma, ret = prologue(geo, proj, conv_w, conv_b, poly, gate_b)
        if memory_state is None:                               # 635-643
            W1 = self.W1_init.float().unsqueeze(0).expand(B, H, D, E).contiguous()
            W2 = self.W2_init.float().unsqueeze(0).expand(B, H, E, D).contiguous()
            memory_state = DeepMemoryState(W1, W2, torch.zeros_like(W1), torch.zeros_like(W2))
        y, st = atlas_scan(q, k, v, alpha, eta, theta, gamma,
                           tuple(s.float().contiguous() for s in memory_state), self.scan_cfg)
        if ret is not None:                                    # 720-722
            y = retrieve_gate(geo, y, ret)
        y = self.c_proj(y.reshape(B, T, H * D).to(x.dtype))    # 724-725
        return y, DeepMemoryState(*st)
