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
