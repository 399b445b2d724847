"""Fused adaLN modulation on sm_100a (replaces kernels/adaln_modulation.py).

Returns (1 + scale_msa, tanh(gate_msa), 1 + scale_mlp, tanh(gate_mlp)) from
the raw [.., 4*dim] output of the adaLN linear (adaln_modulation.py:91-155).
"""

from __future__ import annotations

import torch

from .. import _lib
from .utils import require_bf16


def triton_adaln_modulation(raw: torch.Tensor, dim: int):
    expected_last = 4 * dim
    if raw.shape[-1] != expected_last:
        raise ValueError(
            f"raw.shape[-1] must equal 4 * dim = {expected_last}, got raw.shape={raw.shape}")
    _lib.require_device(raw)
    require_bf16(raw)
    raw = raw.contiguous()
    lead = raw.shape[:-1]
    n_rows = raw.numel() // expected_last
    raw2 = raw.view(n_rows, expected_last)
    outs = [torch.empty(n_rows, dim, dtype=raw.dtype, device=raw.device) for _ in range(4)]
    _lib.call("zib_adaln_modulation", raw2.data_ptr(), expected_last, *[o.data_ptr() for o in outs],
              n_rows, dim, _lib.stream_of(raw))
    return tuple(o.view(*lead, dim) for o in outs)


class TritonAdaLNModulation(torch.nn.Module):
    """Module wrapper (adaln_modulation.py:158-194)."""

    def __init__(self, dim: int) -> None:
        super().__init__()
        self.dim = dim

    def forward(self, raw: torch.Tensor):
        return triton_adaln_modulation(raw, self.dim)

    def extra_repr(self) -> str:
        return f"dim={self.dim}"
