"""Fused RMSNorm + gate + residual on sm_100a (replaces kernels/fused_norm_residual.py).

output = residual + gate * RMSNorm(x, weight, eps), same rounding as the
reference kernel (fused_norm_residual.py:58-73).  A gate that broadcasts per
batch row ([B,1,D], the block's case) is read in place instead of being
expanded to [B*S, D] first (fused_norm_residual.py:104).
"""

from __future__ import annotations

import torch

from .. import _lib
from .utils import check_row_size, require_bf16


def _gate_rows(gate: torch.Tensor, shape: torch.Size) -> tuple[torch.Tensor, int, int]:
    """Return (gate_2d, ld_gate, rows_per_batch) for the kernel's row indexing."""
    n = shape[-1]
    rows = int(torch.Size(shape[:-1]).numel())
    g = gate
    while g.dim() < len(shape):
        g = g.unsqueeze(0)
    if len(shape) == 3 and g.shape[0] == shape[0] and g.shape[1] == 1 and g.shape[2] == n:
        g2 = g.reshape(shape[0], n).contiguous()
        return g2, n, shape[1]
    if all(s == 1 for s in g.shape[:-1]) and g.shape[-1] == n:
        g2 = g.reshape(1, n).contiguous()
        return g2, 0, max(rows, 1)
    g2 = g.expand(shape).contiguous().view(rows, n)
    return g2, n, 1


def triton_fused_norm_gate_residual(x: torch.Tensor, residual: torch.Tensor, gate: torch.Tensor,
                                    weight: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    _lib.require_device(x)
    require_bf16(x, residual, gate)
    shape = x.shape
    n = shape[-1]
    check_row_size(n)
    rows = x.numel() // n
    x2 = x.contiguous().view(rows, n)
    r2 = residual.contiguous().view(rows, n)
    g2, ld_gate, rpb = _gate_rows(gate, shape)
    w = weight.detach().to(torch.float32).contiguous()
    y = torch.empty_like(x2)
    _lib.call("zib_norm_gate_residual", x2.data_ptr(), n, r2.data_ptr(), n, g2.data_ptr(), ld_gate, rpb,
              w.data_ptr(), y.data_ptr(), n, rows, n, float(eps), _lib.stream_of(x))
    return y.view(*shape)
