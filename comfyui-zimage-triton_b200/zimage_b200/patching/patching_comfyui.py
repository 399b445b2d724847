"""Patch a ComfyUI NextDiT (Lumina-2 / Z-Image) model with the sm_100a kernels.

Same surface as ``src/zimage_triton/models/patching_comfyui.py`` of the
reference: RMSNorm modules become ``TritonRMSNorm`` (weight shared,
``_original_module`` kept), ``FeedForward._forward_silu_gating`` becomes the
SwiGLU kernel (``_original_silu_gating`` kept), ``JointAttention.forward`` and
``JointTransformerBlock.forward`` are replaced (``_original_forward`` kept),
and ``apply_triton_kernels_comfyui`` returns the same stats dict.

The block forward has two paths with identical arithmetic:

* fused (all five block linears W8A8+Hadamard, no bias, 128-wide heads, no
  GQA): per block 6 row kernels, 4 tcgen05 GEMMs (w1 and w3 run as one
  3840 -> 2x10240 GEMM: they quantise the same activation, int8_linear.py:129-130)
  and SDPA.  Norm -> modulate -> rotate -> quantise, residual -> norm ->
  modulate -> rotate -> quantise and SwiGLU -> rotate -> quantise each run as
  one pass; QK-norm + RoPE run in place on the QKV GEMM output.
* composed: the reference's sequence of module calls, each on a kernel.
"""

from __future__ import annotations

import logging
import types
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import _lib
from ..kernels.fused_qknorm_rope import qknorm_rope_into, rope_tables
from ..kernels.rms_norm import TritonRMSNorm
from ..kernels.swiglu import triton_swiglu_forward

logger = logging.getLogger(__name__)

# The fused block executor and the composed module path compute the same
# values; tests flip this to compare them.
ENABLE_FUSED_BLOCK = True


def _eps(mod: nn.Module) -> float:
    """getattr(mod, 'eps', 1e-5) or 1e-5 (patching_comfyui.py:157-158, :324-327)."""
    return getattr(mod, "eps", 1e-5) or 1e-5


# ---------------------------------------------------------------------------
# RMSNorm replacement (patching_comfyui.py:31-68)
# ---------------------------------------------------------------------------

def _replace_all_rms_norm_comfyui(model: nn.Module, stats: dict) -> None:
    for name, module in list(model.named_modules()):
        if isinstance(module, TritonRMSNorm):
            continue
        if type(module).__name__ != "RMSNorm":
            continue
        if not hasattr(module, "weight") or module.weight is None:
            continue
        parts = name.split(".")
        parent = model
        for part in parts[:-1]:
            parent = getattr(parent, part)
        attr = parts[-1]
        old = getattr(parent, attr)
        new_norm = TritonRMSNorm(old.weight.shape[0], eps=_eps(old))
        new_norm.weight = old.weight
        new_norm._original_module = old
        setattr(parent, attr, new_norm)
        stats["rms_norm"] += 1


# ---------------------------------------------------------------------------
# FFN SwiGLU (patching_comfyui.py:76-107)
# ---------------------------------------------------------------------------

def _make_ffn_forward_comfyui(ffn: nn.Module):
    def _forward_silu_gating(self, x1: torch.Tensor, x3: torch.Tensor) -> torch.Tensor:
        return triton_swiglu_forward(x1, x3)

    return types.MethodType(_forward_silu_gating, ffn)


def _patch_all_ffn_comfyui(model: nn.Module, stats: dict) -> None:
    for module in model.modules():
        if (type(module).__name__ == "FeedForward" and hasattr(module, "w1") and hasattr(module, "w2")
                and hasattr(module, "w3")):
            if not hasattr(module, "_original_silu_gating"):
                module._original_silu_gating = module._forward_silu_gating
            module._forward_silu_gating = _make_ffn_forward_comfyui(module)
            stats["swiglu"] += 1


# ---------------------------------------------------------------------------
# RoPE tables and attention
# ---------------------------------------------------------------------------

def _convert_rope_matrix_to_complex(freqs_cis: torch.Tensor) -> torch.Tensor:
    """2x2 rotation matrices (b, n, [1,] d//2, 2, 2) -> complex64 (patching_comfyui.py:115-134)."""
    cos = freqs_cis[..., 0, 0]
    sin = freqs_cis[..., 1, 0]
    if cos.ndim == 4 and cos.shape[2] == 1:
        cos = cos.squeeze(2)
        sin = sin.squeeze(2)
    return torch.complex(cos.float(), sin.float())


_TABLE_CACHE: dict = {}
_TABLE_CACHE_SIZE = 8


def _cos_sin(freqs_cis: torch.Tensor, batch: int):
    """(cos, sin, batch_stride) fp32 tables from the 2x2-matrix or complex64 form.

    The blocks of one step receive the same few ``freqs_cis`` tensors (the joint
    sequence, and the image and caption parts for the refiners); each conversion is
    cached on (pointer, shape, version), keeping the last few, so it runs once per step.
    The cached value holds the tensor it was built from, so its memory cannot be
    reused by another tensor with the same key while the entry lives.
    """
    key = (freqs_cis.data_ptr(), tuple(freqs_cis.shape), freqs_cis._version, freqs_cis.dtype, batch,
           freqs_cis.device)
    hit = _TABLE_CACHE.get(key)
    if hit is not None:
        return hit[0]
    if freqs_cis.is_complex():
        fc = freqs_cis
    else:
        fc = _convert_rope_matrix_to_complex(freqs_cis)
    val = rope_tables(fc, batch)
    if len(_TABLE_CACHE) >= _TABLE_CACHE_SIZE:
        _TABLE_CACHE.pop(next(iter(_TABLE_CACHE)))
    _TABLE_CACHE[key] = (val, freqs_cis)
    return val


def _attention_bshd(xq: torch.Tensor, xk: torch.Tensor, xv: torch.Tensor,
                    x_mask: Optional[torch.Tensor]) -> torch.Tensor:
    """SDPA on [B,S,H,d] views -> [B,S,H*d] (stand-in for comfy's optimized_attention_masked,
    patching_comfyui.py:197-205, which resolves to torch SDPA by default)."""
    B, S, H, d = xq.shape
    mask = None
    if x_mask is not None:
        mask = x_mask
        if mask.dim() == 2:
            mask = mask[:, None, None, :]
        elif mask.dim() == 3:
            mask = mask[:, None]
    o = F.scaled_dot_product_attention(xq.transpose(1, 2), xk.transpose(1, 2), xv.transpose(1, 2),
                                       attn_mask=mask)
    return o.transpose(1, 2).reshape(B, S, H * d)


def _make_fused_attention_forward(attn: nn.Module):
    """JointAttention.forward with fused QK-norm + RoPE (patching_comfyui.py:137-209).

    Q and K are normalised and rotated in place inside the fresh QKV output.
    """
    n_heads = attn.n_local_heads
    n_kv = attn.n_local_kv_heads
    head_dim = attn.head_dim
    n_rep = n_heads // n_kv
    split_sizes = [n_heads * head_dim, n_kv * head_dim, n_kv * head_dim]
    qn, kn = attn.q_norm, attn.k_norm
    q_eps, k_eps = _eps(qn), _eps(kn)

    def _forward(self, x: torch.Tensor, x_mask: torch.Tensor, freqs_cis: torch.Tensor,
                 transformer_options: dict = {}) -> torch.Tensor:
        bsz, seqlen, _ = x.shape
        qkv = self.qkv(x)
        xq, xk, xv = torch.split(qkv, split_sizes, dim=-1)
        xq = xq.view(bsz, seqlen, n_heads, head_dim)
        xk = xk.view(bsz, seqlen, n_kv, head_dim)
        xv = xv.view(bsz, seqlen, n_kv, head_dim)
        cos, sin, cs_b = _cos_sin(freqs_cis, bsz)
        qknorm_rope_into(xq, xq, qn.weight.detach().float().contiguous(), cos, sin, cs_b, q_eps)
        qknorm_rope_into(xk, xk, kn.weight.detach().float().contiguous(), cos, sin, cs_b, k_eps)
        if n_rep > 1:
            xk = xk.unsqueeze(3).repeat(1, 1, 1, n_rep, 1).flatten(2, 3)
            xv = xv.unsqueeze(3).repeat(1, 1, 1, n_rep, 1).flatten(2, 3)
        return self.out(_attention_bshd(xq, xk, xv, x_mask))

    return types.MethodType(_forward, attn)


def _make_plain_rope_attention_forward(attn: nn.Module):
    """RoPE-only variant used when fused QK-norm is off (patching_comfyui.py:212-272)."""
    n_heads = attn.n_local_heads
    n_kv = attn.n_local_kv_heads
    head_dim = attn.head_dim
    n_rep = n_heads // n_kv
    split_sizes = [n_heads * head_dim, n_kv * head_dim, n_kv * head_dim]

    def _forward(self, x, x_mask, freqs_cis, transformer_options={}):
        bsz, seqlen, _ = x.shape
        xq, xk, xv = torch.split(self.qkv(x), split_sizes, dim=-1)
        xq = self.q_norm(xq.reshape(bsz, seqlen, n_heads, head_dim))
        xk = self.k_norm(xk.reshape(bsz, seqlen, n_kv, head_dim))
        xv = xv.view(bsz, seqlen, n_kv, head_dim)
        cos, sin, cs_b = _cos_sin(freqs_cis, bsz)
        xq = xq.contiguous()
        xk = xk.contiguous()
        qknorm_rope_into(xq, xq, None, cos, sin, cs_b, 0.0)
        qknorm_rope_into(xk, xk, None, cos, sin, cs_b, 0.0)
        if n_rep > 1:
            xk = xk.unsqueeze(3).repeat(1, 1, 1, n_rep, 1).flatten(2, 3)
            xv = xv.unsqueeze(3).repeat(1, 1, 1, n_rep, 1).flatten(2, 3)
        return self.out(_attention_bshd(xq, xk, xv, x_mask))

    return types.MethodType(_forward, attn)


def _patch_attention_comfyui(model: nn.Module, stats: dict, fused: bool = True) -> None:
    for module in model.modules():
        if type(module).__name__ != "JointAttention" or not hasattr(module, "qkv"):
            continue
        if not hasattr(module, "q_norm") or not hasattr(module.q_norm, "weight"):
            continue
        if not hasattr(module, "_original_forward"):
            module._original_forward = module.forward
        if fused:
            module.forward = _make_fused_attention_forward(module)
            stats["fused_qknorm_rope"] += 1
        else:
            module.forward = _make_plain_rope_attention_forward(module)
            stats["rope_3d"] += 1


# ---------------------------------------------------------------------------
# fused block executor
# ---------------------------------------------------------------------------

def _lin_ok(lin: nn.Module) -> bool:
    return (getattr(lin, "_int8_quantized", False) and getattr(lin, "_int8_use_hadamard", False)
            and getattr(lin, "bias", None) is None and hasattr(lin, "_w_int8") and lin._w_int8.is_cuda)


def _f32(w: torch.Tensor) -> torch.Tensor:
    return w.detach().to(torch.float32).contiguous()


def _bf16_exact(w: torch.Tensor) -> torch.Tensor | None:
    """The norm weight as a contiguous bf16 tensor when every value is a bf16 value (always for
    bf16 parameters), else None: the fused norm kernel's bf16-weight entry gives the same results
    as its fp32 entry for such weights."""
    w = w.detach()
    if w.dtype == torch.bfloat16:
        return w.contiguous()
    h = w.to(torch.bfloat16)
    return h.contiguous() if torch.equal(h.to(w.dtype), w) else None


def _block_cache(block: nn.Module):
    """Per-block tensors of the fused path, or None when the block does not qualify.

    The fused path needs W8A8+Hadamard int8 linears on every projection,
    128-wide heads and an FFN width divisible by the 128-group of the w2
    rotation.
    """
    attn, ff = block.attention, block.feed_forward
    lins = (attn.qkv, attn.out, ff.w1, ff.w2, ff.w3)
    if not all(_lin_ok(l) for l in lins):
        return None
    if attn.head_dim != 128 or attn.n_local_heads != attn.n_local_kv_heads:
        return None
    F_ = ff.w1._w_int8.shape[0]
    if F_ % 128 or ff.w3._w_int8.shape[0] != F_:
        return None
    norms = (block.attention_norm1, block.attention_norm2, block.ffn_norm1, block.ffn_norm2,
             attn.q_norm, attn.k_norm)
    if not all(getattr(n, "weight", None) is not None for n in norms):
        return None
    w13 = _w13_halves(ff)
    key = tuple((n.weight.data_ptr(), n.weight._version) for n in norms) + tuple(
        (l._w_int8.data_ptr(), l._w_int8._version, l._w_scale.data_ptr()) for l in lins)
    c = block.__dict__.get("_zib_cache")
    if c is not None and c["key"] == key:
        return c
    c = {
        "an1": _f32(block.attention_norm1.weight), "an2": _f32(block.attention_norm2.weight),
        "fn1": _f32(block.ffn_norm1.weight), "fn2": _f32(block.ffn_norm2.weight),
        "qn": _f32(attn.q_norm.weight), "kn": _f32(attn.k_norm.weight),
        "an1_h": _bf16_exact(block.attention_norm1.weight), "an2_h": _bf16_exact(block.attention_norm2.weight),
        "fn1_h": _bf16_exact(block.ffn_norm1.weight), "fn2_h": _bf16_exact(block.ffn_norm2.weight),
        "eps_an1": _eps(block.attention_norm1), "eps_an2": _eps(block.attention_norm2),
        "eps_fn1": _eps(block.ffn_norm1), "eps_fn2": _eps(block.ffn_norm2),
        "eps_q": _eps(attn.q_norm), "eps_k": _eps(attn.k_norm),
        "F": F_, "w13": w13, "key": key,
    }
    block.__dict__["_zib_cache"] = c
    return c


def _w13_halves(ff: nn.Module) -> torch.Tensor | None:
    """The [2F, K] int8 tensor whose halves are w1's and w3's ``_w_int8`` (the weight layout of
    zib_gemm_w8a8_swiglu_had_w13), or None when the two weights cannot share one.

    The first call moves both weights into one tensor and makes the modules' buffers views of
    its halves (no second copy of either weight); afterwards the halves are found again as
    long as the buffers stay those views.  In-place writes into the buffers (a LoRA refresh)
    keep the layout.
    """
    w1, w3 = ff.w1._w_int8, ff.w3._w_int8
    F_, K_ = w1.shape
    if (w3.shape != w1.shape or w1.stride(1) != 1 or w3.stride(1) != 1 or w1.stride(0) != K_
            or w3.stride(0) != K_ or K_ % 16 or w1.data_ptr() % 16 or w3.data_ptr() % 16
            or w1.device != w3.device):
        return None
    esz = w1.element_size()
    if w3.data_ptr() == w1.data_ptr() + F_ * K_ * esz and w1._base is not None and w1._base is w3._base:
        base = w1._base
        if base.dim() == 2 and tuple(base.shape) == (2 * F_, K_) and base.data_ptr() == w1.data_ptr():
            return base
    w13 = torch.cat([w1, w3], 0)
    ff.w1._buffers["_w_int8"] = w13[:F_]
    ff.w3._buffers["_w_int8"] = w13[F_:]
    return w13


# Cross-block fusion: a fused block whose successor in the same layer list is also
# fused ends with norm+gate+residual fused to the successor's attention_norm1 +
# modulation + rotation + quantisation, and hands the quantised activations (and the
# successor's adaLN output) over through _HANDOFF.  The successor uses them only if
# its input is exactly the tensor produced (pointer and version) for the same
# adaLN input; anything else in between falls back to the plain path.
ENABLE_BLOCK_HANDOFF = True
_HANDOFF: dict | None = None


# When a list, every fused-path GEMM appends (start_event, end_event, 2*M*N*K,
# entry point name) recorded on its launch stream (the benchmark's roofline figures).
GEMM_EVENTS: list | None = None


def _timed_call(name: str, ops_count: int, *args) -> None:
    ev = GEMM_EVENTS
    if ev is not None:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
    _lib.call(name, *args)
    if ev is not None:
        e1.record()
        ev.append((e0, e1, ops_count, name))


def _gemm(q8, sx, lin_w, lin_s, y, M, N, K, stream):
    _timed_call("zib_gemm_w8a8", 2 * M * N * K, q8.data_ptr(), K, lin_w.data_ptr(), lin_w.stride(0),
                sx.data_ptr(), lin_s.data_ptr(), None, y.data_ptr(), y.stride(0), M, N, K, stream)


def _ngr_entry(D: int, ca: dict, a: str, cb: dict, b: str):
    """Entry point and weights of the fused norm + gate + residual + next norm + quantisation: the
    bf16-weight entry when both norm weights hold bf16 values and the row width is its 3840."""
    wa, wb = ca[a + "_h"], cb[b + "_h"]
    if D == 3840 and wa is not None and wb is not None:
        return "zib_norm_gate_residual_mod_quant_w16", wa, wb
    return "zib_norm_gate_residual_mod_quant", ca[a], cb[b]


def fused_block_forward(block: nn.Module, c: dict, x: torch.Tensor, x_mask, freqs_cis: torch.Tensor,
                        adaln_input: torch.Tensor) -> torch.Tensor:
    """One S3-DiT block on the fused kernels; arithmetic of patching_comfyui.py:340-415."""
    B, S, D = x.shape
    M = B * S
    dev = x.device
    _lib.require_device(x)
    if x.dtype != torch.bfloat16:
        raise ValueError(f"fused block computes in bfloat16; got {x.dtype}")
    x = x.contiguous()
    stream = _lib.stream_of(x)
    bf, i8 = torch.bfloat16, torch.int8
    attn, ff = block.attention, block.feed_forward
    H = attn.n_local_heads
    hd = H * 128
    F_ = c["F"]

    esz = 2  # bf16 bytes
    global _HANDOFF
    h, _HANDOFF = _HANDOFF, None
    if (h is not None and h["block"] is block and h["x"] == (x.data_ptr(), x._version, tuple(x.shape))
            and h["adaln"] == (adaln_input.data_ptr(), adaln_input._version)):
        # the previous block already produced this block's adaLN output and quantised input
        raw, gates, q8, sx = h["raw"], h["gates"], h["q8"], h["sx"]
    else:
        raw, gates = _adaln(block, adaln_input, B, D, stream)
        # attention_norm1 -> *(1+scale_msa) -> rotate -> quantise            (:378)
        q8 = torch.empty(M, D, dtype=i8, device=dev)
        sx = torch.empty(M, dtype=bf, device=dev)
        _lib.call("zib_rmsnorm_mod_quant", x.data_ptr(), D, c["an1"].data_ptr(), raw.data_ptr(), None, raw.stride(0), S,
                  q8.data_ptr(), D, sx.data_ptr(), M, D, float(c["eps_an1"]), 1, stream)
    # QKV projection with per-head Q/K RMSNorm + RoPE in the epilogue     (:180-190)
    nqkv = attn.qkv._w_int8.shape[0]
    qkv = torch.empty(M, nqkv, dtype=bf, device=dev)
    qkv5 = qkv.view(B, S, 3, H, 128)
    xq, xk, xv = qkv5[:, :, 0], qkv5[:, :, 1], qkv5[:, :, 2]
    cos, sin, cs_b = _cos_sin(freqs_cis, B)
    if H % 2 == 0 and nqkv == 3 * hd:
        _timed_call("zib_gemm_w8a8_qk_norm_rope", 2 * M * nqkv * D, q8.data_ptr(), D, attn.qkv._w_int8.data_ptr(),
                    attn.qkv._w_int8.stride(0), sx.data_ptr(), attn.qkv._w_scale.data_ptr(), qkv.data_ptr(), nqkv,
                    M, nqkv, D, c["qn"].data_ptr(), c["kn"].data_ptr(), float(c["eps_q"]), float(c["eps_k"]),
                    cos.data_ptr(), sin.data_ptr(), cs_b, S, H, stream)
    else:  # odd head count: a 256-column tile would straddle two heads
        _gemm(q8, sx, attn.qkv._w_int8, attn.qkv._w_scale, qkv, M, nqkv, D, stream)
        qknorm_rope_into(xq, xq, c["qn"], cos, sin, cs_b, c["eps_q"])
        qknorm_rope_into(xk, xk, c["kn"], cos, sin, cs_b, c["eps_k"])
    o = _attention_bshd(xq, xk, xv, x_mask).reshape(M, hd)                  # :197-205
    # out projection: rotate + quantise + GEMM                            (:207)
    if o.stride(-1) != 1 or o.stride(0) % 8 != 0:
        o = o.contiguous()
    q8o = torch.empty(M, hd, dtype=i8, device=dev)
    sxo = torch.empty(M, dtype=bf, device=dev)
    _lib.call("zib_act_quant", o.data_ptr(), o.stride(0), q8o.data_ptr(), hd, sxo.data_ptr(), None, M, hd, 1,
              stream)
    attn_out = torch.empty(M, D, dtype=bf, device=dev)
    _gemm(q8o, sxo, attn.out._w_int8, attn.out._w_scale, attn_out, M, D, hd, stream)
    # x + g_msa * norm2(attn_out); then ffn_norm1 * (1+scale_mlp) -> quantise   (:386-401)
    x1 = torch.empty(M, D, dtype=bf, device=dev)
    q8f = torch.empty(M, D, dtype=i8, device=dev)
    sxf = torch.empty(M, dtype=bf, device=dev)
    ngr, wa, wb = _ngr_entry(D, c, "an2", c, "fn1")
    _lib.call(ngr, attn_out.data_ptr(), D, x.data_ptr(), D, gates.data_ptr(), gates.stride(0), S, wa.data_ptr(),
              x1.data_ptr(), D, wb.data_ptr(), raw.data_ptr() + 2 * D * esz, None, raw.stride(0), q8f.data_ptr(), D,
              sxf.data_ptr(), M, D, float(c["eps_an2"]), float(c["eps_fn1"]), 1, stream)
    # w1 and w3 GEMMs + SwiGLU + w2-input rotation in one launch, then quantise   (swiglu.py:51-58)
    x_rot = torch.empty(M, F_, dtype=bf, device=dev)
    w13 = c.get("w13")
    if w13 is not None:
        _timed_call("zib_gemm_w8a8_swiglu_had_w13", 2 * M * 2 * F_ * D, q8f.data_ptr(), D, w13.data_ptr(),
                    w13.stride(0), sxf.data_ptr(), ff.w1._w_scale.data_ptr(), ff.w3._w_scale.data_ptr(),
                    x_rot.data_ptr(), F_, M, F_, D, stream)
    else:
        _timed_call("zib_gemm_w8a8_swiglu_had", 2 * M * 2 * F_ * D, q8f.data_ptr(), D, ff.w1._w_int8.data_ptr(),
                    ff.w3._w_int8.data_ptr(), D, sxf.data_ptr(), ff.w1._w_scale.data_ptr(),
                    ff.w3._w_scale.data_ptr(), x_rot.data_ptr(), F_, M, F_, D, stream)
    q8h = torch.empty(M, F_, dtype=i8, device=dev)
    sxh = torch.empty(M, dtype=bf, device=dev)
    _lib.call("zib_act_quant", x_rot.data_ptr(), F_, q8h.data_ptr(), F_, sxh.data_ptr(), None, M, F_, 0, stream)
    ffn_out = torch.empty(M, D, dtype=bf, device=dev)
    _gemm(q8h, sxh, ff.w2._w_int8, ff.w2._w_scale, ffn_out, M, D, F_, stream)
    # x1 + g_mlp * ffn_norm2(ffn_out)                                     (:404-411)
    x2 = torch.empty(M, D, dtype=bf, device=dev)
    nxt = block.__dict__.get("_zib_next")
    cn = _handoff_target(nxt, D)
    if cn is None:
        _lib.call("zib_norm_gate_residual", ffn_out.data_ptr(), D, x1.data_ptr(), D, gates.data_ptr() + D * esz,
                  gates.stride(0), S, c["fn2"].data_ptr(), x2.data_ptr(), D, M, D, float(c["eps_fn2"]), stream)
        return x2.view(B, S, D)
    # ... fused with the next block's attention_norm1 * (1 + its scale_msa) -> rotate -> quantise
    raw_n, gates_n = _adaln(nxt, adaln_input, B, D, stream)
    q8n = torch.empty(M, D, dtype=i8, device=dev)
    sxn = torch.empty(M, dtype=bf, device=dev)
    ngr, wa, wb = _ngr_entry(D, c, "fn2", cn, "an1")
    _lib.call(ngr, ffn_out.data_ptr(), D, x1.data_ptr(), D, gates.data_ptr() + D * esz, gates.stride(0), S,
              wa.data_ptr(), x2.data_ptr(), D, wb.data_ptr(), raw_n.data_ptr(), None, raw_n.stride(0),
              q8n.data_ptr(), D, sxn.data_ptr(), M, D, float(c["eps_fn2"]), float(cn["eps_an1"]), 1, stream)
    out = x2.view(B, S, D)
    _HANDOFF = {"block": nxt, "x": (out.data_ptr(), out._version, tuple(out.shape)),
                "adaln": (adaln_input.data_ptr(), adaln_input._version),
                "raw": raw_n, "gates": gates_n, "q8": q8n, "sx": sxn}
    return out


# All blocks of a block list take their adaLN modulation from the same input, so
# one rotation + quantisation of that input and one GEMM over the stacked int8
# weights give every block's modulation (_AdaLNStack).
ENABLE_ADALN_STACK = True


class _AdaLNStack:
    """The adaLN linears of one block list as a single W8A8 GEMM.

    Column for column the stacked GEMM is each block's own W8A8 linear
    (int8_linear.py:114-138: same quantised input rows, int32 sums, scales and
    bias), so the modulations are identical to the per-block ones.  The blocks'
    int8 weights and scales become row slices of the stack (no second copy); the
    stack is rebuilt if any of them changes.  The first block of the list
    evaluates the stack; the later blocks of the same pass reuse that evaluation
    when they get the same adaLN input tensor (held by reference, so its memory
    cannot be reused by another tensor meanwhile) at the same version.
    """

    def __init__(self, blocks):
        self.blocks = list(blocks)
        self.pos = {id(b): i for i, b in enumerate(self.blocks)}
        self.key = None
        self.memo = None

    def _lins(self):
        lins = []
        for b in self.blocks:
            seq = getattr(b, "adaLN_modulation", None)
            mods = list(seq.children()) if isinstance(seq, nn.Sequential) else []
            if len(mods) != 1:
                return None
            lin = mods[0]
            if not (getattr(lin, "_int8_quantized", False) and hasattr(lin, "_w_int8") and lin._w_int8.is_cuda
                    and lin._w_scale.dtype == torch.bfloat16 and lin.bias is not None
                    and lin.bias.dtype == torch.bfloat16 and lin.bias.is_cuda):
                return None
            lins.append(lin)
        if len({(tuple(l._w_int8.shape), bool(l._int8_use_hadamard)) for l in lins}) != 1:
            return None
        return lins

    @staticmethod
    def _key(lins):
        return tuple((l._w_int8.data_ptr(), l._w_int8._version, l._w_scale.data_ptr(), l._w_scale._version,
                      l.bias.data_ptr(), l.bias._version) for l in lins)

    def _build(self, lins):
        N = lins[0]._w_int8.shape[0]
        w = torch.cat([l._w_int8 for l in lins]).contiguous()
        sw = torch.cat([l._w_scale for l in lins]).contiguous()
        for i, l in enumerate(lins):
            l._buffers["_w_int8"] = w[i * N:(i + 1) * N]
            l._buffers["_w_scale"] = sw[i * N:(i + 1) * N]
        self.w, self.sw = w, sw
        self.bias = torch.cat([l.bias.detach() for l in lins]).contiguous()
        self.N, self.K = N, lins[0]._w_int8.shape[1]
        self.had = bool(lins[0]._int8_use_hadamard)
        self.key = self._key(lins)
        self.memo = None

    def get(self, block: nn.Module, x: torch.Tensor, B: int, D: int, stream):
        """(raw [B, 4D], gates [B, 2, D]) of `block` as strided views, or None (not applicable)."""
        i = self.pos.get(id(block))
        lins = self._lins() if i is not None else None
        if lins is None:
            return None
        if self.key != self._key(lins):
            self._build(lins)
        N, K, L = self.N, self.K, len(self.blocks)
        if (N != 4 * D or x.dtype != torch.bfloat16 or not x.is_cuda or x.dim() != 2
                or tuple(x.shape) != (B, K)):
            return None
        m = self.memo
        # the first block recomputes: one evaluation per pass over the list, never reused
        # by a later forward even when it is given the same input tensor
        if i == 0 or m is None or m[0] is not x or m[1] != x._version:
            x2 = x.contiguous()
            q = torch.empty(B, K, dtype=torch.int8, device=x.device)
            sx = torch.empty(B, dtype=torch.bfloat16, device=x.device)
            _lib.call("zib_act_quant", x2.data_ptr(), K, q.data_ptr(), K, sx.data_ptr(), None, B, K,
                      1 if self.had else 0, stream)
            raw_all = torch.empty(B, L * N, dtype=torch.bfloat16, device=x.device)
            _lib.call("zib_gemm_w8a8", q.data_ptr(), K, self.w.data_ptr(), K, sx.data_ptr(), self.sw.data_ptr(),
                      self.bias.data_ptr(), raw_all.data_ptr(), L * N, B, L * N, K, stream)
            # rows (b, l) of raw_all are consecutive 4D-wide rows: one gates launch for all
            gates_all = torch.empty(B * L, 2, D, dtype=torch.bfloat16, device=x.device)
            _lib.call("zib_adaln_gates", raw_all.data_ptr(), N, gates_all.data_ptr(), B * L, D, stream)
            self.memo = m = (x, x._version, raw_all, gates_all)
        return m[2].view(B, L, N)[:, i], m[3].view(B, L, 2, D)[:, i]


def _adaln(block: nn.Module, adaln_input: torch.Tensor, B: int, D: int, stream):
    """adaLN: raw [B, 4D] and gates [B, 2, D], tanh'd once (patching_comfyui.py:368-372).

    Both may be row-strided views (the stacked evaluation): pass stride(0) as their
    leading dimension.
    """
    st = block.__dict__.get("_zib_adaln_stack") if ENABLE_ADALN_STACK else None
    if st is not None:
        r = st.get(block, adaln_input, B, D, stream)
        if r is not None:
            return r
    raw = block.adaLN_modulation(adaln_input).reshape(B, 4 * D).contiguous()
    gates = torch.empty(B, 2, D, dtype=torch.bfloat16, device=raw.device)
    _lib.call("zib_adaln_gates", raw.data_ptr(), 4 * D, gates.data_ptr(), B, D, stream)
    return raw, gates


def _handoff_target(nxt, D: int):
    """Block cache of the successor if the handoff applies to it, else None."""
    if not (ENABLE_BLOCK_HANDOFF and ENABLE_FUSED_BLOCK) or nxt is None:
        return None
    if not nxt.__dict__.get("_zib_fused_ok", False) or getattr(nxt, "dim", None) != D:
        return None
    return _block_cache(nxt)


def _modulated_norm(norm: nn.Module, x: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """norm(x) * (1 + scale) with one kernel when the norm is a TritonRMSNorm."""
    if isinstance(norm, TritonRMSNorm) and x.dtype == torch.bfloat16 and scale.dtype == torch.bfloat16:
        B, S, D = x.shape
        x2 = x.contiguous()
        sc = scale.reshape(B, D).contiguous()
        y = torch.empty_like(x2)
        _lib.call("zib_rmsnorm_mod", x2.data_ptr(), D, _f32(norm.weight).data_ptr(), sc.data_ptr(), None, D, S,
                  y.data_ptr(), D, B * S, D, float(_eps(norm)), _lib.stream_of(x))
        return y
    return norm(x) * (1 + scale.unsqueeze(1))


def _make_block_forward(block: nn.Module, dim: int, use_adaln: bool, use_fused_nr: bool):
    """Patched JointTransformerBlock.forward (patching_comfyui.py:315-417)."""
    from ..kernels.adaln_modulation import triton_adaln_modulation
    from ..kernels.fused_norm_residual import triton_fused_norm_gate_residual

    an2_w = block.attention_norm2.weight
    an2_eps = _eps(block.attention_norm2)
    fn2_w = block.ffn_norm2.weight
    fn2_eps = _eps(block.ffn_norm2)

    def _forward(self, x: torch.Tensor, x_mask: torch.Tensor, freqs_cis: torch.Tensor,
                 adaln_input: Optional[torch.Tensor] = None, timestep_zero_index=None,
                 transformer_options={}) -> torch.Tensor:
        if timestep_zero_index is not None:  # omni mode (:350-358)
            return self._original_forward(x, x_mask, freqs_cis, adaln_input, timestep_zero_index,
                                          transformer_options)
        assert adaln_input is not None
        if ENABLE_FUSED_BLOCK and not use_adaln and use_fused_nr and x.is_cuda:
            c = _block_cache(self)
            if c is not None:
                return fused_block_forward(self, c, x, x_mask, freqs_cis, adaln_input)

        if use_adaln:
            raw = self.adaLN_modulation(adaln_input)
            s_msa, g_msa, s_mlp, g_mlp = triton_adaln_modulation(raw, dim)
            attn_in = self.attention_norm1(x) * s_msa.unsqueeze(1)
        else:
            s_msa, g_msa, s_mlp, g_mlp = self.adaLN_modulation(adaln_input).chunk(4, dim=1)
            g_msa = g_msa.tanh()
            g_mlp = g_mlp.tanh()
            attn_in = _modulated_norm(self.attention_norm1, x, s_msa)
        attn_out = self.attention(attn_in, x_mask, freqs_cis, transformer_options=transformer_options)
        if use_fused_nr:
            x = triton_fused_norm_gate_residual(attn_out, x, g_msa.unsqueeze(1), an2_w, an2_eps)
        else:
            x = x + g_msa.unsqueeze(1) * self.attention_norm2(attn_out)
        if use_adaln:
            ffn_in = self.ffn_norm1(x) * s_mlp.unsqueeze(1)
        else:
            ffn_in = _modulated_norm(self.ffn_norm1, x, s_mlp)
        ffn_out = self.feed_forward(ffn_in)
        if use_fused_nr:
            x = triton_fused_norm_gate_residual(ffn_out, x, g_mlp.unsqueeze(1), fn2_w, fn2_eps)
        else:
            x = x + g_mlp.unsqueeze(1) * self.ffn_norm2(ffn_out)
        return x

    return types.MethodType(_forward, block)


def _patch_block_forward_comfyui(model: nn.Module, stats: dict, enable_adaln: bool = True,
                                 enable_fused_norm_residual: bool = True) -> None:
    for module in model.modules():
        if type(module).__name__ != "JointTransformerBlock":
            continue
        if not getattr(module, "modulation", False) or not hasattr(module, "dim"):
            continue
        if not hasattr(module, "_original_forward"):
            module._original_forward = module.forward
        module.forward = _make_block_forward(module, module.dim, enable_adaln, enable_fused_norm_residual)
        module.__dict__["_zib_fused_ok"] = (not enable_adaln) and enable_fused_norm_residual
        if enable_adaln:
            stats["adaln_modulation"] += 1
        if enable_fused_norm_residual:
            stats["fused_norm_gate_residual"] += 1
    # successor links inside each block list (plain attributes, not submodules)
    for lst in model.modules():
        if isinstance(lst, nn.ModuleList):
            blocks = [m for m in lst if type(m).__name__ == "JointTransformerBlock"]
            if len(blocks) == len(lst):
                for a, b in zip(blocks, blocks[1:] + [None]):
                    a.__dict__["_zib_next"] = b
                stack = _AdaLNStack(blocks)
                for a in blocks:
                    a.__dict__["_zib_adaln_stack"] = stack


def apply_triton_kernels_comfyui(model: nn.Module, enable_fused_norm: bool = True, enable_swiglu: bool = True,
                                 enable_fused_qknorm_rope: bool = True, enable_fused_adaln: bool = True,
                                 enable_fused_norm_residual: bool = True) -> dict[str, int]:
    """Apply the kernel replacements (patching_comfyui.py:457-517); returns replacement counts."""
    stats: dict[str, int] = {
        "rms_norm": 0,
        "swiglu": 0,
        "rope_3d": 0,
        "fused_qknorm_rope": 0,
        "adaln_modulation": 0,
        "fused_norm_gate_residual": 0,
    }
    if enable_fused_norm:
        _replace_all_rms_norm_comfyui(model, stats)
    if enable_swiglu:
        _patch_all_ffn_comfyui(model, stats)
    _patch_attention_comfyui(model, stats, fused=enable_fused_qknorm_rope)
    if enable_fused_adaln or enable_fused_norm_residual:
        _patch_block_forward_comfyui(model, stats, enable_fused_adaln, enable_fused_norm_residual)
    logger.info("ComfyUI sm_100a patching complete: %s", stats)
    return stats
