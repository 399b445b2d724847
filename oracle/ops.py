"""CPU restatement of every op on the Z-Image W8A8 hot path (TEST INFRASTRUCTURE ONLY).

Only tests, ``__graft_entry__.smoke()`` and the CPU legs of ``bench.py`` use
this module.  All tensors are CPU torch tensors.  Each function cites the
reference file:line it restates (paths relative to the reference project).

Rounding conventions (the reference's, made explicit):

* torch elementwise ops on bf16 compute in fp32 and round once to bf16 (RNE).
* Row reductions (sum of squares) follow one canonical order (``sumsq_rows``):
  fp32 sums over chunks of 8 values, added exactly and rounded once.  The
  reference's Triton ``tl.sum`` uses an implementation-defined tree order, so no
  order is canonical; the CUDA kernels use this one.
* ``rsqrt`` is restated as IEEE ``1 / sqrt(v)`` in fp32: the correctly
  rounded square root, then the correctly rounded reciprocal.  Both are
  formed in fp64 and rounded once to fp32, which is exact for sqrt and
  division (53 >= 2*24 + 2 bits); torch's own fp32 ``sqrt`` on CPU is not
  correctly rounded on every input.  The reference's libdevice ``rsqrt`` is an
  approximation; outputs are compared with tolerances for that reason.
* The Hadamard rotation of activations is restated as the correctly rounded
  bf16 of the exact product ``h * sum(+-x)`` with ``h = bf16(1/sqrt(128))``.
  The reference computes it as a bf16 matmul (``int8_linear.py:124-126``),
  whose fp32 accumulation order is a BLAS detail; ``act_quant_had128_matmul``
  restates that form so tests can measure the (tiny) difference.
* Divisions by the Python scalar 127.0 are true divisions (torch CPU).
"""

from __future__ import annotations

import math

import numpy as np
import torch

GROUP = 128  # int8_linear.py:28 _HADAMARD_GROUP_SIZE

# hadamard.py:40-41: torch.tensor(H_np, float32) / (size ** 0.5); entries are
# +-1 divided by sqrt(128) in fp32.
H_FP32 = float((torch.ones(1, dtype=torch.float32) / (GROUP ** 0.5)).item())
# int8_linear.py:120-123 casts H to the activation dtype (bf16).
H_BF16 = float(torch.tensor(H_FP32, dtype=torch.float32).to(torch.bfloat16).float().item())


# ---------------------------------------------------------------------------
# bit-level helpers
# ---------------------------------------------------------------------------

def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """RNE fp32 -> bf16 on raw bits (finite inputs)."""
    b = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    b = (b + 0x7FFF + ((b >> 16) & 1)) >> 16
    return b.astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def round_f64_to_bf16(v: np.ndarray) -> torch.Tensor:
    """Correctly rounded (single RNE) bf16 of an fp64 value.

    Rounds to fp32 first; when the fp32 value sits exactly on a bf16
    midpoint, the sign of the (exact) fp64 residual decides the direction.
    A midpoint strictly between the exact value and its fp32 rounding cannot
    exist, so this is a single correct rounding.
    """
    v = np.asarray(v, dtype=np.float64)
    f = v.astype(np.float32)
    err = v - f.astype(np.float64)
    bits = f.view(np.uint32).astype(np.uint64)
    tie = ((bits & 0xFFFF) == 0x8000) & (err != 0)
    away = tie & (np.sign(err) == np.sign(f))
    rne = (bits + 0x7FFF + ((bits >> 16) & 1)) >> 16
    trunc = bits >> 16
    out = np.where(tie, np.where(away, trunc + 1, trunc), rne).astype(np.uint16)
    return torch.from_numpy(bf16_bits_to_f32(out).copy()).to(torch.bfloat16)


def bf16(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16)


# ---------------------------------------------------------------------------
# Hadamard (hadamard.py)
# ---------------------------------------------------------------------------

def sylvester_signs(n: int) -> np.ndarray:
    """Sylvester Hadamard sign matrix, H[i, j] = (-1)^popcount(i & j).

    Same ordering as ``scipy.linalg.hadamard`` used by ``hadamard.py:40``.
    """
    if n & (n - 1):
        raise ValueError(f"Hadamard size must be power of 2, got {n}")
    i = np.arange(n)
    pc = np.vectorize(lambda v: bin(v).count("1"))(i[:, None] & i[None, :])
    return np.where(pc % 2 == 0, 1, -1).astype(np.int8)


def fwht_f64(x: np.ndarray) -> np.ndarray:
    """Exact (fp64) unnormalised Walsh-Hadamard transform over the last axis of 128."""
    y = np.array(x, dtype=np.float64, copy=True)
    n = y.shape[-1]
    h = 1
    while h < n:
        y = y.reshape(*y.shape[:-1], n // (2 * h), 2, h)
        a = y[..., 0, :].copy()
        b = y[..., 1, :]
        y = np.stack([a + b, a - b], axis=-2).reshape(*y.shape[:-3], n)
        h *= 2
    return y


def rotate_activation_exact(x: torch.Tensor) -> torch.Tensor:
    """x_rot = bf16( x[m, 128g:128g+128] @ H_bf16 ), exact sum, one rounding.

    Restates ``int8_linear.py:119-126`` / ``hadamard.py:78-107``.
    """
    M, K = x.shape
    if K % GROUP:
        raise ValueError(f"features {K} not divisible by group_size {GROUP}")
    s = fwht_f64(x.float().numpy().reshape(M, K // GROUP, GROUP)) * H_BF16
    return round_f64_to_bf16(s.reshape(M, K))


def rotate_activation_matmul(x: torch.Tensor) -> torch.Tensor:
    """The reference's own form: bf16 batched matmul against H in bf16 (int8_linear.py:124-126)."""
    M, K = x.shape
    H = torch.from_numpy(sylvester_signs(GROUP).astype(np.float32)) * H_FP32
    Hb = H.to(torch.bfloat16)
    return torch.matmul(x.view(M, K // GROUP, GROUP), Hb).reshape(M, K)


# ---------------------------------------------------------------------------
# activation quantisation (int8_linear.py:129-130)
# ---------------------------------------------------------------------------

def quantize_rotated(x_rot: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-token symmetric int8 quantisation of a bf16 row block (int8_linear.py:129-130)."""
    x_scale = x_rot.abs().amax(dim=-1, keepdim=True).clamp(min=1e-5) / 127.0
    x_int8 = (x_rot / x_scale).round().clamp(-128, 127).to(torch.int8)
    return x_int8, x_scale


def act_quant_had128(x: torch.Tensor):
    """Rotate (exact) + quantise: returns (q int8 [M,K], sx bf16 [M,1], x_rot bf16 [M,K])."""
    x_rot = rotate_activation_exact(x)
    q, s = quantize_rotated(x_rot)
    return q, s, x_rot


def act_quant_had128_matmul(x: torch.Tensor):
    x_rot = rotate_activation_matmul(x)
    q, s = quantize_rotated(x_rot)
    return q, s, x_rot


def act_quant_plain(x: torch.Tensor):
    """W8A8 without rotation (int8_linear.py:87-88), used when K % 128 != 0."""
    q, s = quantize_rotated(x)
    return q, s


# ---------------------------------------------------------------------------
# weight prep (hadamard.py:47-75, int8_linear.py:67-73, :256-281)
# ---------------------------------------------------------------------------

def rotate_weight_exact(w: torch.Tensor) -> torch.Tensor:
    """W_rot = W @ H^T per 128-group, in fp64 with the fp32 constant 1/sqrt(128), rounded to fp32."""
    N, K = w.shape
    s = fwht_f64(w.float().numpy().reshape(N, K // GROUP, GROUP)) * np.float64(H_FP32)
    return torch.from_numpy(s.reshape(N, K).astype(np.float32))


def quantize_weight_per_channel(w32: torch.Tensor):
    """int8_linear.py:67-73 (fp32 in, int8 + fp32 scale out)."""
    scale = w32.abs().amax(dim=1).clamp(min=1e-5) / 127.0
    wq = (w32 / scale.unsqueeze(1)).round().clamp(-128, 127).to(torch.int8)
    return wq, scale


def weight_prep(w: torch.Tensor, hadamard: bool = True):
    """Returns (w_int8 [N,K], w_scale bf16 [N], w_scale_fp32 [N])."""
    w32 = rotate_weight_exact(w) if hadamard else w.float()
    wq, s32 = quantize_weight_per_channel(w32)
    return wq, s32.to(torch.bfloat16), s32


# ---------------------------------------------------------------------------
# GEMM + dequant epilogue (int8_linear.py:133-138)
# ---------------------------------------------------------------------------

def gemm_acc_i32(q: torch.Tensor, wq: torch.Tensor) -> torch.Tensor:
    """int32 accumulators acc[m, n] = sum_k q[m,k] * wq[n,k] (torch._int_mm, int8_linear.py:133)."""
    M = q.shape[0]
    if M > 16 and M % 8 == 0 and q.shape[1] % 8 == 0 and wq.shape[0] % 8 == 0:
        return torch._int_mm(q, wq.t())
    return (q.to(torch.int64) @ wq.to(torch.int64).t()).to(torch.int32)


def dequant_epilogue(acc: torch.Tensor, sx: torch.Tensor, sw: torch.Tensor,
                     bias: torch.Tensor | None) -> torch.Tensor:
    """y = bf16(acc) * bf16(sx * sw) (+ bias), all bf16 (int8_linear.py:134-137)."""
    y = acc.to(torch.bfloat16) * (sx.reshape(-1, 1) * sw.reshape(1, -1))
    if bias is not None:
        y = y + bias
    return y


def w8a8_linear(x: torch.Tensor, wq: torch.Tensor, sw: torch.Tensor,
                bias: torch.Tensor | None = None, hadamard: bool = True) -> torch.Tensor:
    """_make_w8a8_hadamard_forward._forward (int8_linear.py:114-138) on a 2-D bf16 input."""
    if hadamard:
        q, sx, _ = act_quant_had128(x)
    else:
        q, sx = act_quant_plain(x)
    return dequant_epilogue(gemm_acc_i32(q, wq), sx, sw, bias)


# ---------------------------------------------------------------------------
# RMSNorm family (rms_norm.py:47-57, fused_norm_residual.py:58-73)
# ---------------------------------------------------------------------------

def sumsq_rows(x: torch.Tensor) -> torch.Tensor:
    """Row sums of squares of a bf16 tensor in the kernels' canonical order, fp32 [..., 1].

    The row is cut into chunks of 8 consecutive values (zero-padded at the end).  Within a
    chunk the even and the odd positions are summed separately in fp32, in order
    (each square of a bf16 value is exact in fp32; every addition rounds once), and the two
    sums are added: s_c = ((x0^2 + x2^2) + x4^2) + x6^2 + (((x1^2 + x3^2) + x5^2) + x7^2).
    The chunk sums are added exactly (fp64; exact while their exponents lie within 29 bits of
    each other) and rounded once to fp32, so the result does not depend on how a kernel
    distributes the chunks over its threads.  The reference's Triton ``tl.sum`` is an fp32
    tree whose order is a compiler detail.
    """
    n = x.shape[-1]
    pad = (-n) % 8
    v = x.float().numpy().astype(np.float32)
    if pad:
        v = np.concatenate([v, np.zeros(v.shape[:-1] + (pad,), np.float32)], -1)
    v = v.reshape(*v.shape[:-1], -1, 8)
    sq = v * v                                   # exact
    e = ((sq[..., 0] + sq[..., 2]) + sq[..., 4]) + sq[..., 6]
    o = ((sq[..., 1] + sq[..., 3]) + sq[..., 5]) + sq[..., 7]
    s = (e + o).astype(np.float64).sum(-1, keepdims=True)
    return torch.from_numpy(s.astype(np.float32))


def rstd_rows(x: torch.Tensor, eps: float) -> torch.Tensor:
    """rsqrt(mean(x^2) + eps) per row in fp32 (canonical chunked sum, IEEE ops)."""
    n = x.shape[-1]
    ss = sumsq_rows(x)
    ms = (ss.double() / n).float()
    sq = torch.sqrt((ms + np.float32(eps)).double()).float()
    return (1.0 / sq.double()).float()


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    """Y = bf16( bf16(x * rstd) * w )  (rms_norm.py:47-57).

    The weight product is formed in fp32 and rounded once to bf16, which equals
    the Triton kernel's result both for bf16 weights (exact fp32 product) and
    for fp32 weights (fp32 product, rounded at the bf16 store).
    """
    shape = x.shape
    x2 = x.reshape(-1, shape[-1])
    xn = (x2.float() * rstd_rows(x2, eps)).to(torch.bfloat16)
    return (xn.float() * w.float()).to(x.dtype).reshape(shape)


def modulate(n: torch.Tensor, scale: torch.Tensor, shift: torch.Tensor | None = None) -> torch.Tensor:
    """n * (1 + scale) per batch row (patching_comfyui.py:378, :401); optional shift (zero = reference).

    n [B, S, D] bf16, scale/shift [B, D] bf16.
    """
    y = n * (1 + scale.unsqueeze(1))
    if shift is not None:
        y = y + shift.unsqueeze(1)
    return y


def fma_bf16(a: torch.Tensor, b: torch.Tensor, c: torch.Tensor) -> torch.Tensor:
    """RN_bf16(a * b + c) of bf16 tensors with one rounding (a bf16 fused multiply-add).

    a * b of two bf16 values is exact in fp64, and so is the sum with a bf16 c
    unless their exponents are more than 37 bits apart, where c (or a*b) alone
    decides the bf16 result; round_f64_to_bf16 then rounds once.
    """
    v = a.double() * b.double() + c.double()
    return round_f64_to_bf16(v.numpy())


def norm_gate_residual(x, residual, gate, w, eps: float = 1e-5):
    """Y = RN_bf16(R + G * bf16(bf16(X * rstd) * W)), one rounding of the gate product and the
    residual add (fused_norm_residual.py:58-73).

    The reference writes ``R_row + G_row * X_scaled`` on bf16 values; the Triton
    compiler contracts the bf16 multiply and add into one fused multiply-add, which
    rounds once (measured against the reference run on a B200: identical on 368,640
    of 368,640 sampled outputs; a separate rounding of the product differs on 17%).
    x, residual [B, S, D]; gate broadcastable [B, 1, D] or [B, D].
    """
    shape = x.shape
    D = shape[-1]
    xs = rms_norm(x, w, eps)
    g = gate.reshape(gate.shape[0], 1, D) if gate.dim() == 2 else gate
    return fma_bf16(g.expand(shape), xs, residual).reshape(shape)


# ---------------------------------------------------------------------------
# fp32 exp / sigmoid / tanh with a fixed operation order
# ---------------------------------------------------------------------------
# exp by Cody & Waite two-constant range reduction (x = k ln2 + r, |r| <= ln2/2)
# and the degree-7 Taylor polynomial of e^r in Horner form with fused
# multiply-adds, then an exact scaling by 2^k; every step is one IEEE fp32
# operation (fma_f32 below restates the fused multiply-add exactly), so this
# restatement and the CUDA kernels produce identical bits.  The reference
# computes these functions with Triton's / torch's own fp32 implementations
# (swiglu.py:55, adaln_modulation.py:73-74, patching_comfyui.py:371-372); all
# agree to a few ulp.

_F = np.float32
EXP_C = [_F(1.98412701e-04), _F(1.38888892e-03), _F(8.33333377e-03), _F(4.16666679e-02),
         _F(1.66666672e-01), _F(0.5), _F(1.0), _F(1.0)]
INV_LN2, LN2_HI, LN2_LO = _F(1.44269502), _F(0.693145751953125), _F(1.42860677e-06)
TANH_C = [_F(-8.86323552e-03), _F(2.18694880e-02), _F(-5.39682545e-02), _F(1.33333340e-01),
          _F(-3.33333343e-01)]


def fma_f32(a, b, c) -> np.ndarray:
    """IEEE fp32 fused multiply-add, RN(a*b + c) with a single rounding.

    a*b is exact in fp64 (2 x 24 significant bits); TwoSum gives prod + c = s + err
    exactly; RN32(s + err) equals RN32(s) unless s is exactly halfway between two
    fp32 values, where the sign of err picks the neighbour.
    """
    a64 = np.asarray(a, dtype=_F).astype(np.float64)
    b64 = np.asarray(b, dtype=_F).astype(np.float64)
    c64 = np.asarray(c, dtype=_F).astype(np.float64)
    prod = a64 * b64
    s = prod + c64
    bb = s - prod
    err = (prod - (s - bb)) + (c64 - bb)
    r = s.astype(_F)
    r64 = r.astype(np.float64)
    other = 2.0 * s - r64                      # the other fp32 neighbour when s is a midpoint
    tie = (s != r64) & (other.astype(_F).astype(np.float64) == other) & (err != 0)
    up = np.maximum(r64, other)
    dn = np.minimum(r64, other)
    fixed = np.where(err > 0, up, dn).astype(_F)
    return np.where(tie, fixed, r).astype(_F)


def exp_f32(x: np.ndarray) -> np.ndarray:
    x = np.minimum(np.maximum(np.asarray(x, dtype=_F), _F(-87.0)), _F(88.0))
    k = np.rint(x * INV_LN2).astype(_F)
    r = fma_f32(-k, LN2_HI, x)
    r = fma_f32(-k, LN2_LO, r)
    p = np.full_like(r, EXP_C[0])
    for c in EXP_C[1:]:
        p = fma_f32(p, r, c)
    return np.ldexp(p.astype(_F), k.astype(np.int32)).astype(_F)


# exp overflows fp32 above this argument (ln of the largest finite fp32, rounded down)
EXP_OVERFLOW = _F(88.72283935546875)


def sigmoid_f32(g: np.ndarray) -> np.ndarray:
    """1 / (1 + exp(-g)); exactly 0 where exp(-g) overflows to inf, as in fp32 arithmetic."""
    g = np.asarray(g, dtype=_F)
    s = (_F(1.0) / (_F(1.0) + exp_f32(-g))).astype(_F)
    return np.where(-g > EXP_OVERFLOW, _F(0.0), s).astype(_F)


def tanh_f32(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=_F)
    a = np.abs(x)
    x2 = (a * a).astype(_F)
    p = np.full_like(a, TANH_C[0])
    for c in TANH_C[1:]:
        p = (p * x2).astype(_F) + c
    small = (a + ((p * x2).astype(_F) * a).astype(_F)).astype(_F)
    e = exp_f32((_F(-2.0) * a).astype(_F))
    big = ((_F(1.0) - e) / (_F(1.0) + e)).astype(_F)
    return np.copysign(np.where(a < _F(0.25), small, big), x).astype(_F)


def _np32(t: torch.Tensor) -> np.ndarray:
    return t.float().numpy()


def tanh_bf16(t: torch.Tensor) -> torch.Tensor:
    """tanh of a bf16 tensor in fp32, rounded once to bf16."""
    return torch.from_numpy(tanh_f32(_np32(t))).to(t.dtype)


# ---------------------------------------------------------------------------
# SwiGLU (swiglu.py:51-58)
# ---------------------------------------------------------------------------

def swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """out = bf16( silu_fp32(gate) ) * up, silu = g * sigmoid(g) in fp32."""
    g = _np32(gate)
    silu = torch.from_numpy((g * sigmoid_f32(g)).astype(_F))
    return silu.to(up.dtype) * up


# ---------------------------------------------------------------------------
# RoPE (rope_3d.py:56-89, fused_qknorm_rope.py:85-151)
# ---------------------------------------------------------------------------

def rope_pairs(xn: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Interleaved-pair rotation in fp32; xn [..., d] bf16; cos/sin [..., d/2] fp32.

    The reference writes ``xe*c - xo*s`` and ``xo*c + xe*s`` (rope_3d.py:80-84,
    fused_qknorm_rope.py:140-141); its compiler contracts the first product with
    the add/subtract into a fused multiply-add: ne = fma(xe, c, -(xo*s)),
    no = fma(xo, c, xe*s) (identical to the reference run on a B200 on every
    sampled output; the uncontracted form differs on 1 in 20,000).
    """
    xe = _np32(xn[..., 0::2])
    xo = _np32(xn[..., 1::2])
    c = np.broadcast_to(cos.float().numpy(), xe.shape)
    s = np.broadcast_to(sin.float().numpy(), xe.shape)
    ne = fma_f32(xe, c, -(xo * s).astype(_F))
    no = fma_f32(xo, c, (xe * s).astype(_F))
    out = np.stack([ne, no], axis=-1).reshape(*xn.shape[:-1], xn.shape[-1])
    return torch.from_numpy(np.ascontiguousarray(out)).to(xn.dtype)


def _cos_sin(freqs_cis: torch.Tensor, batch: int):
    if freqs_cis.shape[0] != batch:
        freqs_cis = freqs_cis.expand(batch, -1, -1)
    return freqs_cis.real.float().unsqueeze(2), freqs_cis.imag.float().unsqueeze(2)


def fused_qknorm_rope(x: torch.Tensor, w: torch.Tensor, freqs_cis: torch.Tensor, eps: float = 1e-5):
    """x [B,S,H,d] bf16; w [d]; freqs_cis complex64 [B or 1, S, d/2] (fused_qknorm_rope.py:85-151)."""
    B, S, H, d = x.shape
    if d % 2:
        raise ValueError(f"head_dim must be even, got {d}")
    if freqs_cis.shape[-1] != d // 2:
        raise ValueError(f"freqs_cis last dim {freqs_cis.shape[-1]} != head_dim//2 {d // 2}")
    xn = rms_norm(x, w, eps)
    c, s = _cos_sin(freqs_cis, B)
    return rope_pairs(xn, c, s)


def rope_3d(x: torch.Tensor, freqs_cis: torch.Tensor) -> torch.Tensor:
    """RoPE only (rope_3d.py:56-89)."""
    B, S, H, d = x.shape
    if d % 2:
        raise ValueError(f"head_dim must be even, got {d}")
    if freqs_cis.shape[-1] != d // 2:
        raise ValueError(f"freqs_cis last dim {freqs_cis.shape[-1]} != head_dim//2 {d // 2}")
    c, s = _cos_sin(freqs_cis, B)
    return rope_pairs(x, c, s)


def convert_rope_matrix_to_complex(freqs_cis: torch.Tensor) -> torch.Tensor:
    """2x2 rotation matrices [..., d/2, 2, 2] -> complex64 (patching_comfyui.py:115-134)."""
    cos = freqs_cis[..., 0, 0]
    sin = freqs_cis[..., 1, 0]
    if cos.ndim == 4 and cos.shape[2] == 1:
        cos = cos.squeeze(2)
        sin = sin.squeeze(2)
    return torch.complex(cos.float(), sin.float())


def rope_angles(positions: torch.Tensor, axes_dims=(32, 48, 48), theta: float = 256.0) -> torch.Tensor:
    """Angles [S, sum(d_i)/2] for multi-axis RoPE: pos_i * theta^(-2j/d_i), fp64 then fp32 trig.

    positions: int [S, n_axes].  Per axis, frequencies are
    theta ** -(2j / d_i) for j < d_i/2, concatenated in axis order.
    """
    parts = []
    for a, d in enumerate(axes_dims):
        j = torch.arange(0, d // 2, dtype=torch.float64)
        omega = 1.0 / (theta ** (2.0 * j / d))
        parts.append(positions[:, a].to(torch.float64)[:, None] * omega[None, :])
    return torch.cat(parts, dim=-1)


def rope_freqs_complex(positions: torch.Tensor, axes_dims=(32, 48, 48), theta: float = 256.0):
    """complex64 [S, d/2] with cos/sin computed in fp64 and rounded to fp32."""
    ang = rope_angles(positions, axes_dims, theta)
    return torch.complex(torch.cos(ang).float(), torch.sin(ang).float())


def rope_freqs_matrix(positions: torch.Tensor, axes_dims=(32, 48, 48), theta: float = 256.0):
    """The same table in the 2x2-matrix form [S, d/2, 2, 2] fp32 ([[c, -s], [s, c]])."""
    fc = rope_freqs_complex(positions, axes_dims, theta)
    c, s = fc.real, fc.imag
    return torch.stack([torch.stack([c, -s], -1), torch.stack([s, c], -1)], -2)


def zimage_positions(grid_h: int = 64, grid_w: int = 64, n_text: int = 512) -> torch.Tensor:
    """(frame, row, col) ids: image tokens on frame 1 over the grid, then text tokens on frames 0..n_text-1."""
    r, c = torch.meshgrid(torch.arange(grid_h), torch.arange(grid_w), indexing="ij")
    img = torch.stack([torch.ones(grid_h * grid_w, dtype=torch.long), r.flatten(), c.flatten()], -1)
    txt = torch.stack([torch.arange(n_text), torch.zeros(n_text, dtype=torch.long),
                       torch.zeros(n_text, dtype=torch.long)], -1)
    return torch.cat([img, txt], 0)


# ---------------------------------------------------------------------------
# adaLN modulation (patching_comfyui.py:368-372; adaln_modulation.py:68-81)
# ---------------------------------------------------------------------------

def adaln_chunks(raw: torch.Tensor, dim: int):
    """Eager default: chunk(4) + tanh on the gates, scales raw (patching_comfyui.py:368-372)."""
    s_msa, g_msa, s_mlp, g_mlp = raw.reshape(raw.shape[0], 4 * dim).chunk(4, dim=1)
    return s_msa, tanh_bf16(g_msa), s_mlp, tanh_bf16(g_mlp)


def adaln_modulation(raw: torch.Tensor, dim: int):
    """Triton variant: (1+scale_msa, tanh(gate_msa), 1+scale_mlp, tanh(gate_mlp)) (adaln_modulation.py:68-81)."""
    if raw.shape[-1] != 4 * dim:
        raise ValueError(f"raw.shape[-1] must equal 4 * dim = {4 * dim}, got raw.shape={raw.shape}")
    lead = raw.shape[:-1]
    r = raw.reshape(-1, 4 * dim)
    sm, gm, sp, gp = r[:, :dim], r[:, dim:2 * dim], r[:, 2 * dim:3 * dim], r[:, 3 * dim:]
    out = (sm + 1.0, tanh_bf16(gm), sp + 1.0, tanh_bf16(gp))
    return tuple(o.reshape(*lead, dim) for o in out)


# ---------------------------------------------------------------------------
# attention (SDPA stand-in for comfy's optimized_attention_masked)
# ---------------------------------------------------------------------------

def sdpa(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """q,k,v [B,S,H,d] bf16 -> [B,S,H*d] bf16; fp32 softmax(QK^T/sqrt(d))V, non-causal."""
    B, S, H, d = q.shape
    o = torch.nn.functional.scaled_dot_product_attention(
        q.float().transpose(1, 2), k.float().transpose(1, 2), v.float().transpose(1, 2))
    return o.transpose(1, 2).reshape(B, S, H * d).to(q.dtype)


__all__ = [n for n in dir() if not n.startswith("_")]
