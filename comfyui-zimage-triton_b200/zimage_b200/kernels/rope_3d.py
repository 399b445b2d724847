"""Interleaved-pair RoPE on sm_100a (replaces kernels/rope_3d.py).

Same aliasing as the reference (rope_3d.py:128-163): the kernel works in
place on ``x.contiguous()``, so a contiguous input is rotated in place and
returned.
"""

from __future__ import annotations

import torch

from .. import _lib
from .fused_qknorm_rope import qknorm_rope_into, rope_tables
from .utils import require_bf16


def triton_rope_3d(x: torch.Tensor, freqs_cis: torch.Tensor) -> torch.Tensor:
    batch, seq, heads, head_dim = x.shape
    half_dim = head_dim // 2
    if head_dim % 2 != 0:
        raise ValueError(f"head_dim must be even, got {head_dim}")
    if freqs_cis.shape[-1] != half_dim:
        raise ValueError(f"freqs_cis last dim {freqs_cis.shape[-1]} != head_dim//2 {half_dim}")
    if head_dim != 128:
        raise ValueError(f"zimage_b200 rope_3d supports head_dim 128, got {head_dim}")
    _lib.require_device(x)
    require_bf16(x)
    cos, sin, cs_b = rope_tables(freqs_cis, batch)
    x = x.contiguous()
    return qknorm_rope_into(x, x, None, cos, sin, cs_b, 0.0)
