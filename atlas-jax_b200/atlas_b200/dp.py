"""Data-parallel plumbing for the scan harness.

The reference's only cross-device operation is one mean of the fp32 parameter
gradients per step (atlas_jax/train.py:150-152, scripts/train_distributed.py:78-79),
after the batch was sharded over the 'data' mesh axis.  Sequences are independent,
so the scan itself needs no exchange; the harness reproduces the step's collective
with one NCCL all-reduce of an fp32 buffer holding exactly the model's parameter
count.
"""

import torch
import torch.distributed as dist


def atlas_param_count(n_layer=12, n_embd=768, n_head=12, memory_expand=4, vocab_size=32768, conv_kernel=4,
                      poly_degree=2, omega_window=16, geglu_ff=True, pad_vocab_to=64):
    """Exact parameter count of the reference Atlas LM (atlas_jax/model.py:271-305,
    Block 39-48, MLP 140-155; AtlasMemoryLayer atlas_jax/memory_layer.py:392-457)."""
    C, H = n_embd, n_head
    D = C // H
    E = memory_expand * D
    di = H * D
    vocab = (vocab_size + pad_vocab_to - 1) // pad_vocab_to * pad_vocab_to
    mem = (3 * C * di              # c_q, c_k, c_v (no bias)          memory_layer.py:422-424
           + di * C                # c_proj                           :425
           + 3 * (di * conv_kernel + di)  # ShortConv weight + bias    :427-429, 309-313
           + 3 * (C * H + H)       # alpha, eta, theta gates (bias)   :431-433
           + (C * H + H if omega_window > 1 else 0)  # gamma gate     :435-438
           + (poly_degree if poly_degree > 0 else 0)  # poly coeffs   :440-444
           + H * D                 # ln_gamma                         :446
           + 2 * H * D * E         # W1_init, W2_init                 :448-452
           + (C * H if H > 1 else 0))  # retrieve gate               :454-457
    if geglu_ff:
        inner = int(C * 4 * 2 / 3)
        mlp = C * inner * 2 + inner * C
    else:
        mlp = C * 4 * C * 2
    return vocab * C * 2 + n_layer * (mem + mlp)   # wte + lm_head + blocks


def init(backend="nccl"):
    """Initialises torch.distributed from the torchrun environment (no-op for one process)."""
    import os
    if int(os.environ.get("WORLD_SIZE", "1")) <= 1:
        return 0, 1
    if not dist.is_initialized():
        if backend == "nccl":
            dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
            dist.init_process_group(backend=backend, device_id=dev)
        else:
            dist.init_process_group(backend=backend)
    return dist.get_rank(), dist.get_world_size()


def allreduce_mean_(buf):
    """In-place mean of the gradient buffer over all ranks (the pmean of train.py:151)."""
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(buf, op=dist.ReduceOp.SUM)
        buf.div_(dist.get_world_size())
    return buf


def max_over_ranks(x):
    """Max of a python float over ranks (device-timed steps: the slowest rank sets the time)."""
    if not (dist.is_initialized() and dist.get_world_size() > 1):
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda" if dist.get_backend() == "nccl" else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
