"""Fused per-head RMSNorm + 3-axis RoPE on sm_100a (replaces kernels/fused_qknorm_rope.py).

The reference's wrapper clones x and expands cos/sin over heads before its
kernel (fused_qknorm_rope.py:206-216); here the kernel reads strided x and a
shared [B or 1, S, d/2] cos/sin table directly and writes a fresh output.
"""

from __future__ import annotations

import torch

from .. import _lib
from .utils import require_bf16


def rope_tables(freqs_cis: torch.Tensor, batch: int) -> tuple[torch.Tensor, torch.Tensor, int]:
    """complex64 [Bf, S, d/2] -> (cos, sin) fp32 contiguous and the batch stride (0 if shared)."""
    if freqs_cis.shape[0] not in (1, batch):
        # the reference's freqs_cis.expand(batch, -1, -1) fails the same way
        raise RuntimeError(
            f"freqs_cis batch {freqs_cis.shape[0]} cannot broadcast to batch {batch}")
    cos = freqs_cis.real.to(torch.float32).contiguous()
    sin = freqs_cis.imag.to(torch.float32).contiguous()
    cs_b = 0 if (freqs_cis.shape[0] == 1 and batch > 1) or batch == 1 else cos.stride(0)
    return cos, sin, cs_b


def qknorm_rope_into(x: torch.Tensor, out: torch.Tensor, weight: torch.Tensor | None,
                     cos: torch.Tensor, sin: torch.Tensor, cs_b: int, eps: float) -> torch.Tensor:
    """Launch the kernel on [B,S,H,128] views (last dim contiguous); out may alias x."""
    B, S, H, d = x.shape
    if x.stride(-1) != 1 or out.stride(-1) != 1:
        raise ValueError("qknorm_rope: last dimension must be contiguous")
    _lib.call("zib_qknorm_rope", x.data_ptr(), x.stride(0), x.stride(1), x.stride(2),
              out.data_ptr(), out.stride(0), out.stride(1), out.stride(2),
              cos.data_ptr(), sin.data_ptr(), cs_b,
              None if weight is None else weight.data_ptr(), B, S, H, d, float(eps),
              _lib.stream_of(x))
    return out


def triton_fused_qknorm_rope(x: torch.Tensor, weight: torch.Tensor, freqs_cis: torch.Tensor,
                             eps: float = 1e-5) -> torch.Tensor:
    """RMSNorm(head) then interleaved RoPE; returns a new [B,S,H,d] tensor (input untouched)."""
    batch, seq, heads, head_dim = x.shape
    half_dim = head_dim // 2
    if head_dim % 2 != 0:
        raise ValueError(f"head_dim must be even, got {head_dim}")
    if freqs_cis.shape[-1] != half_dim:
        raise ValueError(f"freqs_cis last dim {freqs_cis.shape[-1]} != head_dim//2 {half_dim}")
    if head_dim != 128:
        raise ValueError(f"zimage_b200 qknorm_rope supports head_dim 128, got {head_dim}")
    _lib.require_device(x)
    require_bf16(x)
    if x.stride(-1) != 1:
        x = x.contiguous()
    cos, sin, cs_b = rope_tables(freqs_cis, batch)
    out = torch.empty((batch, seq, heads, head_dim), dtype=x.dtype, device=x.device)
    w = weight.detach().to(torch.float32).contiguous()
    return qknorm_rope_into(x, out, w, cos, sin, cs_b, eps)
