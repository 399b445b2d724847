"""SwiGLU on sm_100a (replaces kernels/swiglu.py): out = bf16(bf16(silu(gate)) * up)."""

from __future__ import annotations

import torch

from .. import _lib
from .utils import check_row_size, require_bf16


def triton_swiglu_forward(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """``silu(gate) * up`` in one pass (swiglu.py:62-110); ValueError on shape mismatch."""
    if gate.shape != up.shape:
        raise ValueError(
            f"gate and up must have the same shape, got gate={gate.shape} and up={up.shape}")
    _lib.require_device(gate)
    require_bf16(gate, up)
    shape = gate.shape
    n = shape[-1]
    check_row_size(n)
    g2 = gate.contiguous().view(-1, n)
    u2 = up.contiguous().view(-1, n)
    out = torch.empty_like(g2)
    _lib.call("zib_swiglu", g2.data_ptr(), n, u2.data_ptr(), n, out.data_ptr(), n, g2.shape[0], n,
              _lib.stream_of(gate))
    return out.view(*shape)


class TritonSwiGLU(torch.nn.Module):
    """Drop-in SwiGLU activation module (swiglu.py:113-137)."""

    def forward(self, gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
        return triton_swiglu_forward(gate, up)
