"""Oracle S3-DiT block / step composition (TEST INFRASTRUCTURE ONLY).

Restates the reference's patched ``JointTransformerBlock.forward``
(``src/zimage_triton/models/patching_comfyui.py:340-415``, default node
config: eager adaLN chunk+tanh, fused norm+gate+residual) and the patched
``JointAttention.forward`` (``:171-207``), with the FFN composition
``w2(silu(w1 x) * w3 x)`` (``patching.py:109-112``).  Linear layers are either
W8A8+Hadamard (``int8_linear.py:114-138``) or bf16.

Weights are plain dicts of CPU tensors so the same seeded parameters can be
loaded into the product's module tree.
"""

from __future__ import annotations

import torch

from . import ops

DIM = 3840        # kernels/utils.py:11
FFN_DIM = 10240   # kernels/utils.py:12
HEAD_DIM = 128    # kernels/utils.py:13
N_HEADS = 30      # kernels/utils.py:14
ADALN_DIM = 256


def make_layer_params(gen: torch.Generator, dim=DIM, ffn=FFN_DIM, n_heads=N_HEADS,
                      head_dim=HEAD_DIM, adaln_dim=ADALN_DIM, w_std=0.02):
    """Seeded random-init bf16 parameters of one block (N(0, 0.02) linears, N(1, 0.1) norms)."""
    def lin(o, i):
        return (torch.randn(o, i, generator=gen) * w_std).to(torch.bfloat16)

    def nrm(n):
        return (1.0 + 0.1 * torch.randn(n, generator=gen)).to(torch.bfloat16)

    return {
        "qkv": lin(3 * n_heads * head_dim, dim),
        "out": lin(dim, n_heads * head_dim),
        "w1": lin(ffn, dim),
        "w3": lin(ffn, dim),
        "w2": lin(dim, ffn),
        "adaln_w": lin(4 * dim, adaln_dim),
        "adaln_b": (torch.randn(4 * dim, generator=gen) * w_std).to(torch.bfloat16),
        "q_norm": nrm(head_dim),
        "k_norm": nrm(head_dim),
        "attention_norm1": nrm(dim),
        "attention_norm2": nrm(dim),
        "ffn_norm1": nrm(dim),
        "ffn_norm2": nrm(dim),
    }


QUANT_KEYS = ("qkv", "out", "w1", "w3", "w2")


def prep_layer(p: dict, quant_keys=QUANT_KEYS, quant_adaln: bool = False) -> dict:
    """Weight prep of the oracle: adds '<key>_q' / '<key>_s' for each quantised linear."""
    out = dict(p)
    keys = list(quant_keys) + (["adaln_w"] if quant_adaln else [])
    for k in keys:
        wq, sw, _ = ops.weight_prep(p[k])
        out[k + "_q"] = wq
        out[k + "_s"] = sw
    return out


def linear(p: dict, key: str, x2: torch.Tensor, bias=None) -> torch.Tensor:
    if key + "_q" in p:
        return ops.w8a8_linear(x2, p[key + "_q"], p[key + "_s"], bias)
    y = torch.nn.functional.linear(x2, p[key], bias)
    return y


def block_forward(p: dict, x: torch.Tensor, freqs_cis: torch.Tensor, adaln_input: torch.Tensor,
                  eps: float = 1e-5, qk_eps: float = 1e-5, n_heads=N_HEADS, head_dim=HEAD_DIM,
                  trace: dict | None = None, attn=ops.sdpa) -> torch.Tensor:
    """One patched block forward (patching_comfyui.py:340-415).

    x [B,S,D] bf16; freqs_cis complex64 [B or 1, S, d/2]; adaln_input [B, 256] bf16.
    ``attn(q, k, v) -> [B, S, H*d]`` is the attention (fp32 SDPA by default; tests
    may replay the attention library's recorded outputs instead).
    """
    B, S, D = x.shape
    raw = linear(p, "adaln_w", adaln_input, p["adaln_b"])                    # :368
    s_msa, g_msa, s_mlp, g_mlp = ops.adaln_chunks(raw, D)                    # :368-372
    attn_in = ops.modulate(ops.rms_norm(x, p["attention_norm1"], eps), s_msa)  # :378
    qkv = linear(p, "qkv", attn_in.reshape(B * S, D)).reshape(B, S, -1)      # :180
    hd = n_heads * head_dim
    xq = qkv[..., :hd].reshape(B, S, n_heads, head_dim)
    xk = qkv[..., hd:2 * hd].reshape(B, S, n_heads, head_dim)
    xv = qkv[..., 2 * hd:].reshape(B, S, n_heads, head_dim)
    xq = ops.fused_qknorm_rope(xq, p["q_norm"], freqs_cis, qk_eps)          # :189
    xk = ops.fused_qknorm_rope(xk, p["k_norm"], freqs_cis, qk_eps)          # :190
    o = attn(xq, xk, xv)                                                     # :197-205
    attn_out = linear(p, "out", o.reshape(B * S, hd)).reshape(B, S, D)       # :207
    x = ops.norm_gate_residual(attn_out, x, g_msa, p["attention_norm2"], eps)  # :386-393
    ffn_in = ops.modulate(ops.rms_norm(x, p["ffn_norm1"], eps), s_mlp)      # :401
    f2 = ffn_in.reshape(B * S, D)
    h = ops.swiglu(linear(p, "w1", f2), linear(p, "w3", f2))
    ffn_out = linear(p, "w2", h).reshape(B, S, D)
    x = ops.norm_gate_residual(ffn_out, x, g_mlp, p["ffn_norm2"], eps)      # :404-411
    if trace is not None:
        trace.update(qkv=qkv, attn_out=attn_out, ffn_out=ffn_out, q=xq, k=xk)
    return x


def block_forward_rows(p: dict, x: torch.Tensor, bidx: torch.Tensor, sidx: torch.Tensor,
                       freqs_cis: torch.Tensor, adaln_input: torch.Tensor, attn, eps: float = 1e-5,
                       qk_eps: float = 1e-5, n_heads=N_HEADS, head_dim=HEAD_DIM) -> torch.Tensor:
    """``block_forward`` on a subset of token rows (patching_comfyui.py:340-415).

    Every op of the block except attention works row by row, so a row subset is
    exact given the attention output of those rows.  x [R, D] bf16 are the rows;
    bidx / sidx [R] their batch index (adaLN row) and sequence position (RoPE
    row); ``attn(q, k, v)`` takes the rows' [R, H, d] Q, K, V and returns their
    [R, H*d] attention output.
    """
    R, D = x.shape
    raw = linear(p, "adaln_w", adaln_input, p["adaln_b"])
    s_msa, g_msa, s_mlp, g_mlp = ops.adaln_chunks(raw, D)
    x3 = x.unsqueeze(1)                                                   # [R, 1, D]
    attn_in = ops.modulate(ops.rms_norm(x3, p["attention_norm1"], eps), s_msa[bidx])
    qkv = linear(p, "qkv", attn_in.reshape(R, D))
    hd = n_heads * head_dim
    fc = freqs_cis.reshape(-1, freqs_cis.shape[-2], freqs_cis.shape[-1])
    fc = fc[bidx if fc.shape[0] > 1 else torch.zeros_like(bidx), sidx].unsqueeze(1)   # [R, 1, d/2]
    xq = ops.fused_qknorm_rope(qkv[:, :hd].reshape(R, 1, n_heads, head_dim), p["q_norm"], fc, qk_eps)
    xk = ops.fused_qknorm_rope(qkv[:, hd:2 * hd].reshape(R, 1, n_heads, head_dim), p["k_norm"], fc, qk_eps)
    xv = qkv[:, 2 * hd:].reshape(R, n_heads, head_dim)
    o = attn(xq.reshape(R, n_heads, head_dim), xk.reshape(R, n_heads, head_dim), xv)
    attn_out = linear(p, "out", o.reshape(R, hd)).reshape(R, 1, D)
    x3 = ops.norm_gate_residual(attn_out, x3, g_msa[bidx], p["attention_norm2"], eps)
    ffn_in = ops.modulate(ops.rms_norm(x3, p["ffn_norm1"], eps), s_mlp[bidx]).reshape(R, D)
    h = ops.swiglu(linear(p, "w1", ffn_in), linear(p, "w3", ffn_in))
    ffn_out = linear(p, "w2", h).reshape(R, 1, D)
    return ops.norm_gate_residual(ffn_out, x3, g_mlp[bidx], p["ffn_norm2"], eps).reshape(R, D)


def step_forward(layers: list, x, freqs_cis, adaln_input, eps=1e-5, qk_eps=1e-5, **kw):
    for p in layers:
        x = block_forward(p, x, freqs_cis, adaln_input, eps, qk_eps, **kw)
    return x
