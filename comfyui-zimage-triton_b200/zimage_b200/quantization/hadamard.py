"""Block Walsh-Hadamard rotation helpers (replaces quantization/hadamard.py).

``build_hadamard`` builds the same normalised Sylvester matrix as the
reference (hadamard.py:23-44, ``scipy.linalg.hadamard(n) / sqrt(n)``) without
scipy: H[i, j] = (-1)^popcount(i & j) / sqrt(n).  ``rotate_weight`` and
``rotate_activation`` run on the sm_100a kernels (CUDA tensors only): the
weight rotation is exact and rounded once to fp32, the activation rotation
is exact and rounded once to bf16.
"""

from __future__ import annotations

import torch

from .. import _lib

_HADAMARD_CACHE: dict[tuple[int, str, torch.dtype], torch.Tensor] = {}


def hadamard_signs(size: int) -> torch.Tensor:
    if size <= 0 or size & (size - 1) != 0:
        raise ValueError(f"Hadamard size must be power of 2, got {size}")
    i = torch.arange(size)
    a = i[:, None] & i[None, :]
    parity = torch.zeros_like(a)
    while bool((a != 0).any()):
        parity ^= a & 1
        a = a >> 1
    return 1 - 2 * parity


def build_hadamard(size: int, device: str | torch.device = "cpu",
                   dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Normalised orthogonal Hadamard matrix H (H @ H^T = I), cached per (size, device, dtype)."""
    key = (size, str(device), dtype)
    if key in _HADAMARD_CACHE:
        return _HADAMARD_CACHE[key]
    H = hadamard_signs(size).to(dtype=dtype, device=device) / (size ** 0.5)
    _HADAMARD_CACHE[key] = H
    return H


def rotate_weight(weight: torch.Tensor, H: torch.Tensor | None = None, group_size: int = 128) -> torch.Tensor:
    """W_rot = W @ H_block^T per group of 128 (hadamard.py:47-75); fp32 result."""
    out_f, in_f = weight.shape
    if group_size != 128:
        raise ValueError("zimage_b200 supports group_size 128")
    if in_f % group_size != 0:
        raise ValueError(f"in_features {in_f} not divisible by group_size {group_size}")
    _lib.require_device(weight)
    w = weight.detach().to(torch.bfloat16).contiguous()
    if not torch.equal(w.float(), weight.detach().float()):
        raise ValueError("rotate_weight expects bf16-representable weights")
    wq = torch.empty(out_f, in_f, dtype=torch.int8, device=w.device)
    sw = torch.empty(out_f, dtype=torch.bfloat16, device=w.device)
    rot = torch.empty(out_f, in_f, dtype=torch.float32, device=w.device)
    _lib.call("zib_weight_prep", w.data_ptr(), in_f, wq.data_ptr(), in_f, sw.data_ptr(), None,
              rot.data_ptr(), in_f, out_f, in_f, 1, _lib.stream_of(w))
    return rot


def rotate_activation(x: torch.Tensor, H: torch.Tensor | None = None, group_size: int = 128) -> torch.Tensor:
    """x_rot = x @ H_block per group of 128 (hadamard.py:78-107), bf16 result."""
    features = x.shape[-1]
    if group_size != 128:
        raise ValueError("zimage_b200 supports group_size 128")
    if features % group_size != 0:
        raise ValueError(f"features {features} not divisible by group_size {group_size}")
    _lib.require_device(x)
    if x.dtype != torch.bfloat16:
        raise ValueError(f"rotate_activation computes in bfloat16; got {x.dtype}")
    x2 = x.contiguous().view(-1, features)
    M = x2.shape[0]
    q = torch.empty(M, features, dtype=torch.int8, device=x.device)
    sx = torch.empty(M, dtype=torch.bfloat16, device=x.device)
    xr = torch.empty(M, features, dtype=torch.bfloat16, device=x.device)
    _lib.call("zib_act_quant", x2.data_ptr(), features, q.data_ptr(), features, sx.data_ptr(),
              xr.data_ptr(), M, features, 1, _lib.stream_of(x))
    return xr.view(x.shape)
