"""RMSNorm on sm_100a (replaces kernels/rms_norm.py of the reference).

``triton_rms_norm`` / ``TritonRMSNorm`` keep the reference's names and
semantics: y = bf16( bf16(x * rsqrt(mean(x^2) + eps)) * w ), fp32 inside
(rms_norm.py:47-57, :62-102, :105-134).
"""

from __future__ import annotations

import torch

from .. import _lib
from .utils import check_row_size, require_bf16


def _f32(w: torch.Tensor) -> torch.Tensor:
    return w.detach().to(torch.float32).contiguous()


def triton_rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    """RMSNorm over the last dimension; same shape and dtype as ``x``."""
    _lib.require_device(x)
    require_bf16(x)
    shape = x.shape
    n = shape[-1]
    check_row_size(n)
    x2 = x.contiguous().view(-1, n)
    y = torch.empty_like(x2)
    w = _f32(weight)
    _lib.call("zib_rms_norm", x2.data_ptr(), n, w.data_ptr(), y.data_ptr(), n, x2.shape[0], n,
              float(eps), _lib.stream_of(x))
    return y.view(*shape)


class TritonRMSNorm(torch.nn.Module):
    """Drop-in RMSNorm module (rms_norm.py:105-134): shares ``weight``, exposes ``eps``."""

    def __init__(self, hidden_size: int, eps: float = 1e-5) -> None:
        super().__init__()
        self.hidden_size = hidden_size
        self.eps = eps
        self.weight = torch.nn.Parameter(torch.ones(hidden_size))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return triton_rms_norm(x, self.weight, self.eps)

    def extra_repr(self) -> str:
        return f"hidden_size={self.hidden_size}, eps={self.eps}"
