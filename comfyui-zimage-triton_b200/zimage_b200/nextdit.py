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

import math

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
        if not self.modulation:  # context refiner blocks: no adaLN, plain pre/post-norm residuals
            x = x + self.attention_norm2(self.attention(self.attention_norm1(x), x_mask, freqs_cis,
                                                        transformer_options=transformer_options))
            return x + self.ffn_norm2(self.feed_forward(self.ffn_norm1(x)))
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


class TimestepEmbedder(nn.Module):
    """Sinusoidal features of the (scaled) flow time -> Linear -> SiLU -> Linear (the DiT
    timestep embedding): cos/sin of t * 10000^(-j/half), j < half, concatenated."""

    def __init__(self, out_dim: int = 256, freq_dim: int = 256, mid_dim: int = 1024, device=None, dtype=None):
        super().__init__()
        kw = dict(device=device, dtype=dtype)
        self.freq_dim = freq_dim
        self.mlp = nn.Sequential(nn.Linear(freq_dim, mid_dim, bias=True, **kw), nn.SiLU(),
                                 nn.Linear(mid_dim, out_dim, bias=True, **kw))

    def forward(self, t: torch.Tensor) -> torch.Tensor:
        half = self.freq_dim // 2
        j = torch.arange(half, device=t.device, dtype=torch.float32)
        args = t.float()[:, None] * torch.exp(j * (-math.log(10000.0) / half))[None, :]
        emb = torch.cat([torch.cos(args), torch.sin(args)], dim=-1)
        return self.mlp(emb.to(self.mlp[0].weight.dtype if self.mlp[0].weight.is_floating_point()
                               else torch.bfloat16))


class FinalLayer(nn.Module):
    """LayerNorm (no affine) -> * (1 + scale) from the adaLN input -> Linear to patch pixels."""

    def __init__(self, dim: int, out_dim: int, adaln_dim: int = 256, device=None, dtype=None):
        super().__init__()
        kw = dict(device=device, dtype=dtype)
        self.norm_final = nn.LayerNorm(dim, elementwise_affine=False, eps=1e-6, **kw)
        self.linear = nn.Linear(dim, out_dim, bias=True, **kw)
        self.adaLN_modulation = nn.Sequential(nn.SiLU(), nn.Linear(min(dim, adaln_dim), dim, bias=True, **kw))

    def forward(self, x: torch.Tensor, c: torch.Tensor) -> torch.Tensor:
        scale = self.adaLN_modulation(c)
        return self.linear(self.norm_final(x) * (1 + scale.unsqueeze(1)))


class ZImageDiT(nn.Module):
    """The whole Z-Image S3-DiT forward around the main block stack, random-init.

    latents [B, C, H, W] -> 2x2 patches -> x_embedder; caption features [B, L, cap_dim] ->
    cap_embedder (RMSNorm + Linear); flow time -> t_embedder -> the 256-d adaLN input;
    noise_refiner blocks (with adaLN) over the image tokens and context_refiner blocks
    (without) over the caption tokens; then the joint sequence [image tokens, caption
    tokens] through the main ``layers``; final_layer on the image tokens -> velocity
    [B, C, H, W].  RoPE positions: image tokens (frame 1, row, col), caption tokens
    (frame 0 .. L-1, 0, 0), axes (32, 48, 48), theta 256.  Module and attribute names
    are the ones the node's patching and the INT8 layer policy read.
    """

    def __init__(self, n_layers: int = 30, n_refiner_layers: int = 2, dim: int = 3840, n_heads: int = 30,
                 ffn_dim: int = 10240, in_channels: int = 16, patch_size: int = 2, cap_feat_dim: int = 2560,
                 adaln_dim: int = 256, norm_eps: float = 1e-5, qk_norm_eps: float = 1e-5,
                 t_scale: float = 1000.0, axes_dims=(32, 48, 48), rope_theta: float = 256.0,
                 device=None, dtype=torch.bfloat16):
        super().__init__()
        kw = dict(device=device, dtype=dtype)
        self.dim, self.in_channels, self.patch_size = dim, in_channels, patch_size
        self.t_scale, self.axes_dims, self.rope_theta = t_scale, tuple(axes_dims), rope_theta
        self.compute_dtype = dtype
        pix = patch_size * patch_size * in_channels
        self.x_embedder = nn.Linear(pix, dim, bias=True, **kw)
        self.t_embedder = TimestepEmbedder(min(dim, adaln_dim), 256, 1024, **kw)
        self.cap_embedder = nn.Sequential(RMSNorm(cap_feat_dim, norm_eps, **kw), nn.Linear(cap_feat_dim, dim, bias=True, **kw))

        def blocks(n, modulation, base=0):
            return nn.ModuleList([JointTransformerBlock(base + i, dim, n_heads, ffn_dim, norm_eps, qk_norm_eps,
                                                        adaln_dim, modulation=modulation, **kw) for i in range(n)])

        self.noise_refiner = blocks(n_refiner_layers, True)
        self.context_refiner = blocks(n_refiner_layers, False)
        self.layers = blocks(n_layers, True)
        self.final_layer = FinalLayer(dim, pix, adaln_dim, **kw)
        self._rope_cache: dict = {}

    def rope_table(self, gh: int, gw: int, n_text: int, device) -> torch.Tensor:
        """[1, gh*gw + n_text, d/2, 2, 2] fp32 on `device`, built once per resolution."""
        key = (gh, gw, n_text, str(device))
        t = self._rope_cache.get(key)
        if t is None:
            t = rope_freqs_matrix(zimage_positions(gh, gw, n_text), self.axes_dims, self.rope_theta).unsqueeze(0)
            t = self._rope_cache[key] = t.to(device)
        return t

    def forward(self, x: torch.Tensor, timesteps: torch.Tensor, cap_feats: torch.Tensor, x_mask=None,
                transformer_options={}) -> torch.Tensor:
        """x [B, C, H, W] latents; timesteps [B] flow time in [0, 1]; cap_feats [B, L, cap_dim]."""
        B, C, H, W = x.shape
        p = self.patch_size
        gh, gw = H // p, W // p
        n_img = gh * gw
        dt = self.compute_dtype
        img = x.to(dt).reshape(B, C, gh, p, gw, p).permute(0, 2, 4, 3, 5, 1).reshape(B, n_img, p * p * C)
        adaln = self.t_embedder(timesteps * self.t_scale)
        xi = self.x_embedder(img)
        cap = self.cap_embedder(cap_feats.to(dt))
        freqs = self.rope_table(gh, gw, cap.shape[1], x.device)
        f_img, f_txt = freqs[:, :n_img], freqs[:, n_img:]
        for blk in self.noise_refiner:
            xi = blk(xi, None, f_img, adaln_input=adaln, transformer_options=transformer_options)
        for blk in self.context_refiner:
            cap = blk(cap, None, f_txt, transformer_options=transformer_options)
        h = torch.cat([xi, cap], dim=1)
        for blk in self.layers:
            h = blk(h, None, freqs, adaln_input=adaln, transformer_options=transformer_options)
        out = self.final_layer(h[:, :n_img], adaln)
        out = out.reshape(B, gh, gw, p, p, C).permute(0, 5, 1, 3, 2, 4).reshape(B, C, H, W)
        return out.to(x.dtype)


def zimage_positions(grid_h: int = 64, grid_w: int = 64, n_text: int = 512) -> torch.Tensor:
    """Position ids [S, 3] (frame, row, col): image tokens on frame 1 over a grid_h x grid_w
    grid (row-major), then text tokens on frames 0 .. n_text-1 with row = col = 0."""
    r, c = torch.meshgrid(torch.arange(grid_h), torch.arange(grid_w), indexing="ij")
    img = torch.stack([torch.ones(grid_h * grid_w, dtype=torch.long), r.flatten(), c.flatten()], -1)
    txt = torch.stack([torch.arange(n_text), torch.zeros(n_text, dtype=torch.long),
                       torch.zeros(n_text, dtype=torch.long)], -1)
    return torch.cat([img, txt], 0)


def rope_freqs_complex(positions: torch.Tensor, axes_dims=(32, 48, 48), theta: float = 256.0,
                       device=None) -> torch.Tensor:
    """Multi-axis RoPE table, complex64 [S, sum(axes_dims)/2] (cos + i sin).

    Axis a with d_a dimensions contributes d_a/2 rotation pairs with angles
    pos_a * theta^(-2j/d_a), j < d_a/2, concatenated in axis order (Z-Image: frame,
    row, col with (32, 48, 48) and theta 256).  Angles and their cos/sin are formed
    in fp64 on the host and rounded once to fp32, so the table does not depend on
    the device it is used on.
    """
    pos = positions.detach().to("cpu", torch.float64)
    parts = []
    for a, d in enumerate(axes_dims):
        j = torch.arange(0, d // 2, dtype=torch.float64)
        parts.append(pos[:, a, None] * (1.0 / theta ** (2.0 * j / d))[None, :])
    ang = torch.cat(parts, dim=-1)
    fc = torch.complex(torch.cos(ang).float(), torch.sin(ang).float())
    return fc if device is None else fc.to(device)


def rope_freqs_matrix(positions: torch.Tensor, axes_dims=(32, 48, 48), theta: float = 256.0,
                      device=None) -> torch.Tensor:
    """The same table in ComfyUI's 2x2 rotation-matrix form [S, d/2, 2, 2] fp32, [[c, -s], [s, c]]
    (the form ``_convert_rope_matrix_to_complex``, patching_comfyui.py:115-134, reads)."""
    fc = rope_freqs_complex(positions, axes_dims, theta)
    c, s = fc.real, fc.imag
    m = torch.stack([torch.stack([c, -s], -1), torch.stack([s, c], -1)], -2)
    return m if device is None else m.to(device)


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
    norms = {id(m.weight) for m in model.modules() if isinstance(m, RMSNorm)}
    for name, prm in model.named_parameters():
        if id(prm) in norms or name.endswith("norm.weight") or "_norm" in name.split(".")[-2]:
            prm.copy_(1.0 + 0.1 * torch.randn(prm.shape, generator=g, device=dev))
        else:
            prm.copy_(torch.randn(prm.shape, generator=g, device=dev) * w_std)
