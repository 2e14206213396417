"""Shared seeded input recipes and comparison helpers for the tests."""
import numpy as np
import torch


def headed_bf16(B, H, T, d=64, seed=0, f_mode="sigmoid"):
    """Config-2 recipe: q,k,v ~ N(0,1) (k L2-normalised), f = sigmoid(N(2,1)),
    generated on the CPU, q/k/v rounded to bf16."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, T, d, generator=g)
    k = torch.randn(B, H, T, d, generator=g)
    k = k / k.norm(dim=-1, keepdim=True)
    v = torch.randn(B, H, T, d, generator=g)
    x = torch.randn(B, H, T, generator=g)
    if f_mode == "sigmoid":
        f = torch.sigmoid(x + 2.0)
    elif f_mode == "ones":
        f = torch.ones(B, H, T)
    elif f_mode == "zeros":
        f = torch.zeros(B, H, T)
    elif f_mode == "mixed":
        f = torch.sigmoid(x + 2.0)
        f[..., ::7] = 0.0
        f[..., 3::11] = 1.0
        f[..., 5::13] = 1e-3
    else:
        raise ValueError(f_mode)
    return q.bfloat16(), k.bfloat16(), v.bfloat16(), f.float()


def as64(*ts):
    return [t.detach().cpu().double().numpy() for t in ts]


def rel_max_err(a, b):
    """max|a - b| / max|b| (b is the reference)."""
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def rel_fro_err(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
