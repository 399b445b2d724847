"""Shared test helpers: seeded inputs, comparison metrics, the Z-Image-named module tree."""

from __future__ import annotations

import torch
import torch.nn as nn


def seeded_x(M: int, K: int, seed: int = 0, outlier_frac: float = 0.01, outlier_scale: float = 20.0,
             std: float = 1.0) -> torch.Tensor:
    """bf16 [M, K] ~ N(0, std) with a seeded 1% of channels scaled (the W8A8 benchmark input)."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g) * std
    n_out = max(1, int(round(K * outlier_frac)))
    idx = torch.randperm(K, generator=g)[:n_out]
    x[:, idx] *= outlier_scale
    return x.to(torch.bfloat16)


def seeded_w(N: int, K: int, seed: int = 1, std: float = 0.02) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(N, K, generator=g) * std).to(torch.bfloat16)


def rel_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    a = a.double().flatten()
    b = b.double().flatten()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def max_abs(a: torch.Tensor, b: torch.Tensor) -> float:
    return float((a.double() - b.double()).abs().max())


def mismatch(a: torch.Tensor, b: torch.Tensor) -> int:
    return int((a != b).sum())


def ztree():
    """Z-Image-named module tree at tiny width (same as tests/golden/make_golden.py)."""
    from zimage_b200.nextdit import NextDiT

    class ZTree(nn.Module):
        def __init__(self):
            super().__init__()
            d = 128
            self.x_embedder = nn.Linear(64, d)
            self.t_embedder = nn.Sequential(nn.Linear(256, 256), nn.SiLU(), nn.Linear(256, 256))
            self.cap_embedder = nn.Sequential(nn.LayerNorm(256), nn.Linear(256, d))
            m = NextDiT(n_layers=6, dim=d, n_heads=1, ffn_dim=256, adaln_dim=256, dtype=torch.float32)
            self.layers = m.layers
            self.noise_refiner = NextDiT(n_layers=2, dim=d, n_heads=1, ffn_dim=256, dtype=torch.float32).layers
            self.context_refiner = NextDiT(n_layers=2, dim=d, n_heads=1, ffn_dim=256, dtype=torch.float32).layers
            self.final_layer = nn.Sequential(nn.Linear(d, 64))

    torch.manual_seed(0)
    return ZTree()


def midpoint_rows(n_pool: int = 4096, K: int = 3840, seed: int = 11, n_rows: int = 48):
    """Rows of a seeded pool whose rotation reaches the exact-residual rounding path.

    Returns (x, tie_mask): up to ``n_rows`` rows whose fp32 rotation product
    p = fwht(x) * bf16(1/sqrt(128)) sits exactly on a bf16 midpoint (low 16 bits 0x8000),
    where rounding p to bf16 would differ from rounding the exact product; tie_mask
    marks those positions.
    """
    import numpy as np

    from oracle import ops

    x = seeded_x(n_pool, K, seed=seed)
    v = ops.fwht_f64(x.float().numpy().reshape(n_pool, K // 128, 128)).reshape(n_pool, K)
    p = v.astype(np.float32) * np.float32(ops.H_BF16)
    tie = (p.view(np.uint32) & 0xFFFF) == 0x8000
    rows = np.flatnonzero(tie.any(1))[:n_rows]
    return x[torch.from_numpy(rows)], torch.from_numpy(tie[rows])
