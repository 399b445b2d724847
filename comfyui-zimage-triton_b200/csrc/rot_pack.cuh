// Packed-pair (sm_100 f32x2) forms of the per-chunk rotation, rounding and
// int8 quantisation shared by the warp-per-row kernels and the SwiGLU GEMM
// epilogue.  A chunk is 16 bytes = 8 bf16 held by one lane; a 128-element
// Hadamard group is one chunk in each of 16 consecutive lanes.
//
// Every value is the one the scalar forms produce: each packed add, sub, mul
// or fma rounds each of its two fp32 lanes once, exactly like the scalar
// instruction (no packed product feeds a packed add or sub here: the
// assembler may contract such a pair into one fma even with explicit
// rounding modifiers, so those sums stay scalar), the butterflies run in the same order on the same operands
// (index bits 0, 1, 2 in-thread, then 3..6 over xor shuffles), and the
// rounding points are those of int8_linear.py:119-130 (rotation rounded once
// to bf16, x_scale = bf16(bf16(amax) / 127), q = clamp(rne(bf16(x / x_scale)))).
// The packing only removes instructions: two fp32 lanes per arithmetic
// instruction, the first butterfly taken straight from the bf16 pair, three
// 16-bit-pair compares per chunk for the midpoint check, and one saturating
// pack per two int8 outputs.
#pragma once

#include "zib_common.cuh"

namespace zib {
namespace px {

typedef unsigned long long f2;  // two fp32: low word = even element, high word = odd element

__device__ __forceinline__ f2 mk(float lo, float hi) {
  f2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void split(f2 v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ f2 add(f2 a, f2 b) {
  f2 r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ f2 sub(f2 a, f2 b) {
  f2 r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ f2 mul(f2 a, f2 b) {
  f2 r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ f2 fma(f2 a, f2 b, f2 c) {
  f2 r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
// the low 16 bits of both lanes of v, low lane in the low half
__device__ __forceinline__ uint32_t low_halves(f2 v) {
  float lo, hi;
  split(v, lo, hi);
  return __byte_perm(__float_as_uint(lo), __float_as_uint(hi), 0x5410);
}
// round both lanes to bf16 (RNE), packed (low lane in the low half)
__device__ __forceinline__ uint32_t to_bf16x2(f2 v) {
  float lo, hi;
  split(v, lo, hi);
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ f2 from_bf16x2(uint32_t w) {
  return mk(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
}

// acc + v^2 for the bf16 value v, one rounding (mixed-precision fma: no unpacking)
__device__ __forceinline__ float sq_acc(unsigned short v, float acc) {
  asm("fma.rn.f32.bf16 %0, %1, %1, %0;" : "+f"(acc) : "h"(v));
  return acc;
}
// chunk_sumsq (zib_common.cuh) of the chunk's 8 packed bf16 values: even positions are the
// low halves, odd positions the high halves
__device__ __forceinline__ float sumsq_chunk_f32(const uint4& d) {
  float e = 0.0f, o = 0.0f;
  e = sq_acc((unsigned short)(d.x & 0xFFFFu), e);
  o = sq_acc((unsigned short)(d.x >> 16), o);
  e = sq_acc((unsigned short)(d.y & 0xFFFFu), e);
  o = sq_acc((unsigned short)(d.y >> 16), o);
  e = sq_acc((unsigned short)(d.z & 0xFFFFu), e);
  o = sq_acc((unsigned short)(d.z >> 16), o);
  e = sq_acc((unsigned short)(d.w & 0xFFFFu), e);
  o = sq_acc((unsigned short)(d.w >> 16), o);
  return __fadd_rn(e, o);
}
// the same chunk sum widened for the row's exact fp64 accumulation
__device__ __forceinline__ double sumsq_chunk(const uint4& d) { return (double)sumsq_chunk_f32(d); }

// bf16(bf16(v * rstd) * w) of the chunk's 8 bf16 values, w = the chunk's 8
// fp32 weights (rms_norm.py:53-57)
__device__ __forceinline__ uint4 norm_w(const uint4& d, float rstd, const float4& wa, const float4& wb) {
  const f2 W[4] = {mk(wa.x, wa.y), mk(wa.z, wa.w), mk(wb.x, wb.y), mk(wb.z, wb.w)};
  const f2 RS = mk(rstd, rstd);
  const uint32_t v[4] = {d.x, d.y, d.z, d.w};
  uint32_t o[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) o[k] = to_bf16x2(mul(from_bf16x2(to_bf16x2(mul(from_bf16x2(v[k]), RS))), W[k]));
  return make_uint4(o[0], o[1], o[2], o[3]);
}

__device__ __forceinline__ uint4 norm_w(const uint4& d, float rstd, const float* __restrict__ w) {
  return norm_w(d, rstd, __ldg(reinterpret_cast<const float4*>(w)), __ldg(reinterpret_cast<const float4*>(w + 4)));
}

// bf16(bf16(v * rstd) * w) with the chunk's 8 weights as bf16 values: their product with a bf16
// value is exact in fp32, so one packed bf16 multiply (one rounding of the exact product) gives
// the result of norm_w on the same weights held as fp32
__device__ __forceinline__ uint4 norm_w16(const uint4& d, float rstd, const uint4& w) {
  const f2 RS = mk(rstd, rstd);
  const uint32_t v[4] = {d.x, d.y, d.z, d.w}, wv[4] = {w.x, w.y, w.z, w.w};
  uint32_t o[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t n = to_bf16x2(mul(from_bf16x2(v[k]), RS));
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(o[k]) : "r"(n), "r"(wv[k]));
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// zib_expf on both lanes: the same clamp, range reduction, Horner steps and
// exponent insertion, each packed operation rounding each lane once
__device__ __forceinline__ f2 exp_pair(f2 x) {
  float x0, x1;
  split(x, x0, x1);
  x0 = fminf(fmaxf(x0, -87.0f), 88.0f);
  x1 = fminf(fmaxf(x1, -87.0f), 88.0f);
  x = mk(x0, x1);
  // scalar product and sum: a packed mul feeding a packed add may be contracted
  // into one fma by the assembler, which would change the rounding
  const f2 t = mk(__fadd_rn(__fmul_rn(x0, kInvLn2), 12582912.0f), __fadd_rn(__fmul_rn(x1, kInvLn2), 12582912.0f));
  const f2 k = sub(t, mk(12582912.0f, 12582912.0f));
  f2 r = fma(k, mk(-kLn2Hi, -kLn2Hi), x);  // (-k) ln2hi + x
  r = fma(k, mk(-kLn2Lo, -kLn2Lo), r);
  f2 p = fma(mk(kExpC7, kExpC7), r, mk(kExpC6, kExpC6));
  p = fma(p, r, mk(kExpC5, kExpC5));
  p = fma(p, r, mk(kExpC4, kExpC4));
  p = fma(p, r, mk(kExpC3, kExpC3));
  p = fma(p, r, mk(0.5f, 0.5f));
  p = fma(p, r, mk(1.0f, 1.0f));
  p = fma(p, r, mk(1.0f, 1.0f));
  float t0, t1, p0, p1;
  split(t, t0, t1);
  split(p, p0, p1);
  // (ki << 23) == (bits(t) << 23) mod 2^32: the shifter's bits vanish in the shift
  return mk(__uint_as_float(__float_as_uint(p0) + (__float_as_uint(t0) << 23)),
            __uint_as_float(__float_as_uint(p1) + (__float_as_uint(t1) << 23)));
}

// RN(1/d), d >= 1: Markstein's method (P. Markstein, "Computation of elementary functions on the
// IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990): the hardware reciprocal
// approximation r0 (within one ulp) corrected once with the exact residual e = 1 - d r0 (an fma)
// as r0 + r0 e (an fma, one rounding).  Reciprocals below the normal range take the IEEE
// reciprocal.  Equal to it on every d the SiLU forms (checked exhaustively over all bf16 gates).
__device__ __forceinline__ float rcp_rn_pos(float d) {
  if (!(d < 8.50705917e37f)) return __frcp_rn(d);  // 2^126: 1/d would leave the normal range
  float r0;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r0) : "f"(d));
  return __fmaf_rn(r0, __fmaf_rn(-d, r0, 1.0f), r0);
}

// g * sigmoid(g) in fp32 of the bf16 pair g2 (swiglu.py:51-55), sigmoid = the
// correctly rounded reciprocal of 1 + exp(-g), 0 where exp(-g) overflows fp32
__device__ __forceinline__ f2 silu_f32x2(uint32_t g2) {
  const f2 g = from_bf16x2(g2);
  const f2 e = exp_pair(mul(g, mk(-1.0f, -1.0f)));
  float d0, d1, g0, g1;
  split(add(mk(1.0f, 1.0f), e), d0, d1);
  split(g, g0, g1);
  const float s0 = -g0 > kExpOverflow ? 0.0f : rcp_rn_pos(d0);
  const float s1 = -g1 > kExpOverflow ? 0.0f : rcp_rn_pos(d1);
  return mul(g, mk(s0, s1));
}

// bf16(g * sigmoid(g)) of the bf16 pair g2
__device__ __forceinline__ uint32_t silu_bf16x2(uint32_t g2) { return to_bf16x2(silu_f32x2(g2)); }

// (a + b, a - b) for the bf16 pair w = (a low, b high), each rounded once to fp32
__device__ __forceinline__ f2 bfly0(uint32_t w) {
  const float b = __uint_as_float(w & 0xFFFF0000u);
  const unsigned short a = (unsigned short)(w & 0xFFFFu);
  float s, d;
  asm("add.rn.f32.bf16 %0, %1, %2;" : "=f"(s) : "h"(a), "f"(b));
  asm("sub.rn.f32.bf16 %0, %1, %2;" : "=f"(d) : "h"(a), "f"(b));
  return mk(s, d);
}

// Unnormalised Walsh-Hadamard transform over 128 of chunk d (index bits 0..2)
// and the same chunk of the 15 other lanes of its half-warp (bits 3..6).
// P[k] = elements (2k, 2k+1).  Every lane of the warp must call this.
__device__ __forceinline__ void fwht128(const uint4& d, f2 P[4], int lane) {
  P[0] = bfly0(d.x);
  P[1] = bfly0(d.y);
  P[2] = bfly0(d.z);
  P[3] = bfly0(d.w);
  const f2 t0 = add(P[0], P[1]), t1 = sub(P[0], P[1]);  // bit 1
  const f2 t2 = add(P[2], P[3]), t3 = sub(P[2], P[3]);
  P[0] = add(t0, t2);                                    // bit 2
  P[2] = sub(t0, t2);
  P[1] = add(t1, t3);
  P[3] = sub(t1, t3);
#pragma unroll
  for (int m = 1; m < 16; m <<= 1) {  // bits 3..6: v' = o + v (lower lane) or o - v (upper)
    const float sg = (lane & m) ? -1.0f : 1.0f;
    const f2 SG = mk(sg, sg);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float lo, hi;
      split(P[k], lo, hi);
      const float olo = __shfl_xor_sync(0xFFFFFFFFu, lo, m);
      const float ohi = __shfl_xor_sync(0xFFFFFFFFu, hi, m);
      P[k] = fma(P[k], SG, mk(olo, ohi));
    }
  }
}

// The same transform with two chunks per lane: A = chunk i and B = chunk i + 8
// of a 128-group (index bit 6 tells them apart) held by 8 consecutive lanes
// (bits 3..5).  Bits 0..2 in-thread on each chunk, bits 3..5 over xor shuffles
// (m = 1, 2, 4), bit 6 in-thread between A and B: the stages, operands and
// order of fwht128, with three shuffle stages instead of four.  Every lane of
// the warp must call this.
__device__ __forceinline__ void fwht128_pair(const uint4& a, const uint4& b, f2 A[4], f2 B[4], int lane) {
  const uint32_t wa[4] = {a.x, a.y, a.z, a.w}, wb[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    A[k] = bfly0(wa[k]);
    B[k] = bfly0(wb[k]);
  }
  {
    const f2 t0 = add(A[0], A[1]), t1 = sub(A[0], A[1]), t2 = add(A[2], A[3]), t3 = sub(A[2], A[3]);
    A[0] = add(t0, t2);
    A[2] = sub(t0, t2);
    A[1] = add(t1, t3);
    A[3] = sub(t1, t3);
  }
  {
    const f2 t0 = add(B[0], B[1]), t1 = sub(B[0], B[1]), t2 = add(B[2], B[3]), t3 = sub(B[2], B[3]);
    B[0] = add(t0, t2);
    B[2] = sub(t0, t2);
    B[1] = add(t1, t3);
    B[3] = sub(t1, t3);
  }
#pragma unroll
  for (int m = 1; m < 8; m <<= 1) {
    const float sg = (lane & m) ? -1.0f : 1.0f;
    const f2 SG = mk(sg, sg);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float lo, hi;
      split(A[k], lo, hi);
      float olo = __shfl_xor_sync(0xFFFFFFFFu, lo, m);
      float ohi = __shfl_xor_sync(0xFFFFFFFFu, hi, m);
      A[k] = fma(A[k], SG, mk(olo, ohi));
      split(B[k], lo, hi);
      olo = __shfl_xor_sync(0xFFFFFFFFu, lo, m);
      ohi = __shfl_xor_sync(0xFFFFFFFFu, hi, m);
      B[k] = fma(B[k], SG, mk(olo, ohi));
    }
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) {  // bit 6: A + B (lower), A - B (upper)
    const f2 s = add(A[k], B[k]);
    B[k] = sub(A[k], B[k]);
    A[k] = s;
  }
}

// bf16 chunk of the correctly rounded products P * bf16(1/sqrt(128)).  The
// fp32 product rounded to bf16 is the correct rounding unless it sits exactly
// on a bf16 midpoint (low 16 bits 0x8000); if any lane of the warp has one,
// the warp takes the exact residual path for its whole chunk.  Every lane of
// the warp must call this.
__device__ __forceinline__ uint4 had_round(const f2 P[4]) {
  const f2 H = mk(kHBf16, kHBf16);
  f2 Q[4];
  uint32_t y[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    Q[k] = mul(P[k], H);
    y[k] = low_halves(Q[k]) ^ 0x80008000u;  // a zero half marks a midpoint
  }
  const uint32_t m = __vminu2(__vimin3_u16x2(y[0], y[1], y[2]), y[3]);
  const bool tie = (m & 0xFFFFu) == 0u || m < 0x10000u;
  if (__any_sync(0xFFFFFFFFu, tie)) {
    uint32_t w[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float lo, hi;
      split(P[k], lo, hi);
      const float a = mul_round_bf16(lo, kHBf16), b = mul_round_bf16(hi, kHBf16);
      w[k] = (__float_as_uint(a) >> 16) | (__float_as_uint(b) & 0xFFFF0000u);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
  }
  return make_uint4(to_bf16x2(Q[0]), to_bf16x2(Q[1]), to_bf16x2(Q[2]), to_bf16x2(Q[3]));
}

// Running |max| of bf16 chunks as bit patterns: the signed 16-bit maximum
// tracks the largest positive value, the unsigned one the largest negative
// magnitude (sign bit set sorts above every positive pattern).
struct AbsMax {
  uint32_t s = 0x80008000u, u = 0u;
  __device__ __forceinline__ void add(const uint4& d) {
    s = __vimax3_s16x2(s, d.x, d.y);
    s = __vimax3_s16x2(s, d.z, d.w);
    u = __vimax3_u16x2(u, d.x, d.y);
    u = __vimax3_u16x2(u, d.z, d.w);
  }
  // |max| bit patterns of the two half-lanes, packed (as the bf16x2 absmax)
  __device__ __forceinline__ uint32_t packed() const { return __vmaxu2(__vmaxs2(s, 0u), u & 0x7FFF7FFFu); }
};

__device__ __forceinline__ int cvt_rni_bf16(uint32_t h16) {
  int r;
  asm("cvt.rni.s32.bf16 %0, %1;" : "=r"(r) : "h"((unsigned short)h16));
  return r;
}
// bytes (b, a) saturated to int8 in the low 16 bits, c in the high 16 bits
__device__ __forceinline__ uint32_t pack_s8(int a, int b, uint32_t c) {
  uint32_t r;
  asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}

// int8 of the chunk's 8 bf16 values: clamp(rne(bf16(v / s)), -128, 127)
// (int8_linear.py:130), with v / s formed as RN(v * RN(1/s)).  That equals
// RN(v / s) after the bf16 rounding for every bf16 v and bf16 s: with 8-bit
// significands, v / s = (m_v / m_s) 2^k is never a bf16 midpoint (a midpoint
// needs an odd 9-bit numerator) and stays at least 2^15 / 255 > 128 fp32 ulps
// away from every midpoint, while the reciprocal form is within 2 ulps of the
// quotient (checked exhaustively over all bf16 v for 1024 scales by the CPU
// tests).  The saturating pack clamps to [-128, 127].
__device__ __forceinline__ uint2 quant_chunk(const uint4& d, float rcp) {
  const f2 R = mk(rcp, rcp);
  const uint32_t w[4] = {d.x, d.y, d.z, d.w};
  int q[8];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t b = to_bf16x2(mul(from_bf16x2(w[k]), R));
    q[2 * k] = cvt_rni_bf16(b & 0xFFFFu);
    q[2 * k + 1] = cvt_rni_bf16(b >> 16);
  }
  return make_uint2(pack_s8(q[1], q[0], pack_s8(q[3], q[2], 0u)),
                    pack_s8(q[5], q[4], pack_s8(q[7], q[6], 0u)));
}

// quant_chunk for a row whose |max| is finite (every bf16(v / s) finite, |v / s| < 2^22):
// rne to an integer by one packed fp32 add of 1.5 * 2^23 (the sum's unit in the last place is 1,
// so the add rounds v / s to the nearest integer, ties to even, exactly like cvt.rni), whose
// low bits, less those of 1.5 * 2^23, are the integer; two values per add instead of one
// conversion each on the narrow conversion pipe.
__device__ __forceinline__ uint2 quant_chunk_rne(const uint4& d, float rcp) {
  constexpr float kRne = 12582912.0f;  // 1.5 * 2^23
  constexpr int kRneBits = 0x4B400000;
  const f2 R = mk(rcp, rcp), M = mk(kRne, kRne);
  const uint32_t w[4] = {d.x, d.y, d.z, d.w};
  int q[8];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t b = to_bf16x2(mul(from_bf16x2(w[k]), R));
    float lo, hi;
    split(add(from_bf16x2(b), M), lo, hi);
    q[2 * k] = __float_as_int(lo) - kRneBits;
    q[2 * k + 1] = __float_as_int(hi) - kRneBits;
  }
  return make_uint2(pack_s8(q[1], q[0], pack_s8(q[3], q[2], 0u)),
                    pack_s8(q[5], q[4], pack_s8(q[7], q[6], 0u)));
}

}  // namespace px
}  // namespace zib
