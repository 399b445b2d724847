"""A NextDiT-shaped module tree for running the patched path without ComfyUI.

ComfyUI (``comfy.ldm.lumina.model``) is not a dependency of this package.
This module restates the parts of its Z-Image transformer that the patch
surface touches - class names ``JointTransformerBlock``, ``JointAttention``,
``FeedForward``, ``RMSNorm`` and the attribute names the reference reads
(``patching_comfyui.py:137-449``, ``int8_linear.py:27-64``) - with random-init
weights, so the node, the tests and the benchmark have a model to patch.
Its unpatched forwards are plain eager torch; after ``ZImageTritonApply``
every hot op runs on the sm_100a kernels.

Sizes default to Z-Image: dim 3840, 30 heads x 128, FFN 10240, adaLN input 256.
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float = 1e-5, device=None, dtype=None):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim, device=device, dtype=dtype))

    def forward(self, x):
        xf = x.float()
        n = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)).to(x.dtype)
        return (n.float() * self.weight.float()).to(x.dtype)


def _rope_2x2(x: torch.Tensor, freqs_cis: torch.Tensor) -> torch.Tensor:
    """Interleaved-pair rotation with the [..., d/2, 2, 2] matrix form."""
    B, S, H, d = x.shape
    f = freqs_cis
    if f.dim() == 6:
        f = f.squeeze(2)
    xr = x.float().reshape(B, S, H, d // 2, 1, 2)
    f = f.reshape(f.shape[0], S, 1, d // 2, 2, 2)
    out = (f[..., 0] * xr[..., 0] + f[..., 1] * xr[..., 1])
    return out.reshape(B, S, H, d).to(x.dtype)


class JointAttention(nn.Module):
    def __init__(self, dim: int, n_heads: int, n_kv_heads: int | None = None, qk_norm: bool = True,
                 eps: float = 1e-5, device=None, dtype=None):
        super().__init__()
        self.n_kv_heads = n_kv_heads or n_heads
        self.n_local_heads = n_heads
        self.n_local_kv_heads = self.n_kv_heads
        self.n_rep = self.n_local_heads // self.n_local_kv_heads
        self.head_dim = dim // n_heads
        kw = dict(device=device, dtype=dtype)
        self.qkv = nn.Linear(dim, (n_heads + 2 * self.n_kv_heads) * self.head_dim, bias=False, **kw)
        self.out = nn.Linear(n_heads * self.head_dim, dim, bias=False, **kw)
        if qk_norm:
            self.q_norm = RMSNorm(self.head_dim, eps, **kw)
            self.k_norm = RMSNorm(self.head_dim, eps, **kw)
        else:
            self.q_norm = self.k_norm = nn.Identity()

    def forward(self, x, x_mask, freqs_cis, transformer_options={}):
        B, S, _ = x.shape
        hd = self.n_local_heads * self.head_dim
        kd = self.n_local_kv_heads * self.head_dim
        xq, xk, xv = torch.split(self.qkv(x), [hd, kd, kd], dim=-1)
        xq = self.q_norm(xq.reshape(B, S, self.n_local_heads, self.head_dim))
        xk = self.k_norm(xk.reshape(B, S, self.n_local_kv_heads, self.head_dim))
        xv = xv.reshape(B, S, self.n_local_kv_heads, self.head_dim)
        xq, xk = _rope_2x2(xq, freqs_cis), _rope_2x2(xk, freqs_cis)
        if self.n_rep > 1:
            xk = xk.repeat_interleave(self.n_rep, dim=2)
            xv = xv.repeat_interleave(self.n_rep, dim=2)
        o = F.scaled_dot_product_attention(xq.transpose(1, 2), xk.transpose(1, 2), xv.transpose(1, 2))
        return self.out(o.transpose(1, 2).reshape(B, S, hd))


class FeedForward(nn.Module):
    def __init__(self, dim: int, hidden_dim: int, device=None, dtype=None):
        super().__init__()
        kw = dict(device=device, dtype=dtype)
        self.w1 = nn.Linear(dim, hidden_dim, bias=False, **kw)
        self.w2 = nn.Linear(hidden_dim, dim, bias=False, **kw)
        self.w3 = nn.Linear(dim, hidden_dim, bias=False, **kw)

    def _forward_silu_gating(self, x1, x3):
        return F.silu(x1) * x3

    def forward(self, x):
        return self.w2(self._forward_silu_gating(self.w1(x), self.w3(x)))


class JointTransformerBlock(nn.Module):
    def __init__(self, layer_id: int, dim: int, n_heads: int, ffn_dim: int, norm_eps: float = 1e-5,
                 qk_norm_eps: float = 1e-5, adaln_dim: int = 256, modulation: bool = True,
                 device=None, dtype=None):
        super().__init__()
        kw = dict(device=device, dtype=dtype)
        self.dim = dim
        self.layer_id = layer_id
        self.modulation = modulation
        self.attention = JointAttention(dim, n_heads, eps=qk_norm_eps, **kw)
        self.feed_forward = FeedForward(dim, ffn_dim, **kw)
        self.attention_norm1 = RMSNorm(dim, norm_eps, **kw)
        self.ffn_norm1 = RMSNorm(dim, norm_eps, **kw)
        self.attention_norm2 = RMSNorm(dim, norm_eps, **kw)
        self.ffn_norm2 = RMSNorm(dim, norm_eps, **kw)
        if modulation:
            self.adaLN_modulation = nn.Sequential(nn.Linear(min(dim, adaln_dim), 4 * dim, bias=True, **kw))

    def forward(self, x, x_mask, freqs_cis, adaln_input=None, timestep_zero_index=None,
                transformer_options={}):
        s_msa, g_msa, s_mlp, g_mlp = self.adaLN_modulation(adaln_input).chunk(4, dim=1)
        g_msa, g_mlp = g_msa.tanh(), g_mlp.tanh()
        x = x + g_msa.unsqueeze(1) * self.attention_norm2(
            self.attention(self.attention_norm1(x) * (1 + s_msa.unsqueeze(1)), x_mask, freqs_cis,
                           transformer_options=transformer_options))
        x = x + g_mlp.unsqueeze(1) * self.ffn_norm2(
            self.feed_forward(self.ffn_norm1(x) * (1 + s_mlp.unsqueeze(1))))
        return x


class NextDiT(nn.Module):
    """The main-layer stack of the Z-Image S3-DiT (30 blocks at full size)."""

    def __init__(self, n_layers: int = 30, dim: int = 3840, n_heads: int = 30, ffn_dim: int = 10240,
                 norm_eps: float = 1e-5, qk_norm_eps: float = 1e-5, adaln_dim: int = 256,
                 device=None, dtype=torch.bfloat16):
        super().__init__()
        self.dim = dim
        self.layers = nn.ModuleList([
            JointTransformerBlock(i, dim, n_heads, ffn_dim, norm_eps, qk_norm_eps, adaln_dim,
                                  device=device, dtype=dtype) for i in range(n_layers)])

    def forward(self, x, adaln_input, freqs_cis, x_mask=None, transformer_options={}):
        for layer in self.layers:
            x = layer(x, x_mask, freqs_cis, adaln_input=adaln_input, transformer_options=transformer_options)
        return x


LINEAR_KEYS = {
    "qkv": ("attention", "qkv"), "out": ("attention", "out"), "w1": ("feed_forward", "w1"),
    "w2": ("feed_forward", "w2"), "w3": ("feed_forward", "w3"),
}
NORM_KEYS = {
    "q_norm": ("attention", "q_norm"), "k_norm": ("attention", "k_norm"),
    "attention_norm1": ("attention_norm1",), "attention_norm2": ("attention_norm2",),
    "ffn_norm1": ("ffn_norm1",), "ffn_norm2": ("ffn_norm2",),
}


def _get(mod, path):
    for p in path:
        mod = getattr(mod, p)
    return mod


@torch.no_grad()
def load_layer_params(block: JointTransformerBlock, p: dict) -> None:
    """Copy a dict of per-block tensors (keys as in LINEAR_KEYS / NORM_KEYS, plus
    'adaln_w' / 'adaln_b') into a block's parameters."""
    for k, path in LINEAR_KEYS.items():
        _get(block, path).weight.copy_(p[k])
    for k, path in NORM_KEYS.items():
        _get(block, path).weight.copy_(p[k])
    block.adaLN_modulation[0].weight.copy_(p["adaln_w"])
    block.adaLN_modulation[0].bias.copy_(p["adaln_b"])


@torch.no_grad()
def random_init_(model: NextDiT, seed: int = 0, w_std: float = 0.02) -> None:
    """Seeded init on the model's device: N(0, w_std) linears and biases, N(1, 0.1) norm weights."""
    dev = next(model.parameters()).device
    g = torch.Generator(device=dev).manual_seed(seed)
    for name, prm in model.named_parameters():
        if name.endswith("norm.weight") or "_norm" in name.split(".")[-2]:
            prm.copy_(1.0 + 0.1 * torch.randn(prm.shape, generator=g, device=dev))
        else:
            prm.copy_(torch.randn(prm.shape, generator=g, device=dev) * w_std)
