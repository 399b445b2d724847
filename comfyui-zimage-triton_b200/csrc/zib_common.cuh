// Shared device/host helpers for the Z-Image B200 kernels (sm_100a only).
//
// Rounding helpers restate the reference's bf16 rounding points
// (src/zimage_triton/quantization/int8_linear.py:114-138 and the Triton
// kernels under src/zimage_triton/kernels/): every elementwise bf16 op is an
// fp32 op rounded once to bf16 (RNE).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/zimage_b200.h"

#define ZIB_HOST_CHECK(cond, status, ...)             \
  do {                                                \
    if (!(cond)) {                                    \
      zib_set_error(__VA_ARGS__);                     \
      return (status);                                \
    }                                                 \
  } while (0)

// thread-local last-error message (defined in zib_api.cu)
void zib_set_error(const char* fmt, ...);
int zib_check_launch(const char* what);

namespace zib {

constexpr int kGroup = 128;                      // Hadamard block (int8_linear.py:28)
constexpr float kHBf16 = 0.08837890625f;         // bf16(1/sqrt(128)), int8_linear.py:120-123
constexpr float kHFp32 = 0.0883883461356163f;    // fp32 1/sqrt(128), hadamard.py:40-41

__device__ __forceinline__ float bf16_round(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}

// RN_bf16(a * b + c) with one rounding (fma.rn.bf16) of bf16-representable a, b, c:
// the bf16 multiply-add that the reference's Triton kernels contract
// (fused_norm_residual.py:69-73)
__device__ __forceinline__ float bf16_fma(float a, float b, float c) {
  const unsigned short ha = (unsigned short)(__float_as_uint(a) >> 16);
  const unsigned short hb = (unsigned short)(__float_as_uint(b) >> 16);
  const unsigned short hc = (unsigned short)(__float_as_uint(c) >> 16);
  unsigned short hd;
  asm("fma.rn.bf16 %0, %1, %2, %3;" : "=h"(hd) : "h"(ha), "h"(hb), "h"(hc));
  return __uint_as_float((uint32_t)hd << 16);
}

// Canonical sum of squares of one chunk of 8 consecutive row values (bf16-representable
// floats): the even and the odd positions are summed in order in fp32 (each square is exact,
// each addition rounds once) and the two sums added.  Rows add their chunk sums exactly (fp64,
// exact while the chunk sums' exponents lie within 29 bits of each other) and round once, so
// the result does not depend on how a kernel spreads the chunks over threads.
__device__ __forceinline__ float chunk_sumsq(const float v[8]) {
  float e = __fmul_rn(v[0], v[0]), o = __fmul_rn(v[1], v[1]);
  e = __fmaf_rn(v[2], v[2], e);
  o = __fmaf_rn(v[3], v[3], o);
  e = __fmaf_rn(v[4], v[4], e);
  o = __fmaf_rn(v[5], v[5], o);
  e = __fmaf_rn(v[6], v[6], e);
  o = __fmaf_rn(v[7], v[7], o);
  return __fadd_rn(e, o);
}

__device__ __forceinline__ float bf16_bits_to_float(uint16_t b) {
  return __uint_as_float(((uint32_t)b) << 16);
}

__device__ __forceinline__ uint16_t float_to_bf16_bits(float v) {
  __nv_bfloat16 h = __float2bfloat16_rn(v);
  return *reinterpret_cast<uint16_t*>(&h);
}

// Correctly rounded bf16 of the exact product s * h, given fp32 s.
// p = RN32(s*h); e = s*h - p exactly (FMA).  A bf16 midpoint strictly between
// s*h and p cannot exist, so only p sitting exactly on a midpoint needs the
// sign of e to pick the direction.
__device__ __forceinline__ float mul_round_bf16(float s, float h) {
  float p = __fmul_rn(s, h);
  float e = __fmaf_rn(s, h, -p);
  uint32_t b = __float_as_uint(p);
  if ((b & 0xFFFFu) == 0x8000u && e != 0.0f) {
    uint32_t t = b & 0xFFFF0000u;
    bool away = (e > 0.0f) == (p > 0.0f);
    return __uint_as_float(away ? t + 0x10000u : t);
  }
  return bf16_round(p);
}

// q = clamp(rne(bf16(v / s)), -128, 127) for bf16-valued v and scale s
// (int8_linear.py:130).  v / s is formed as v * rcp with rcp = RN(1/s); that
// product is within 2 ulp of RN(v/s), so the bf16 rounding can only differ when
// the product's low 16 bits are within a few ulp of the bf16 midpoint 0x8000;
// those (rare) lanes recompute the quotient with an IEEE division.
__device__ __forceinline__ int quant_i8(float v, float s, float rcp) {
  float q0 = __fmul_rn(v, rcp);
  uint32_t lo = __float_as_uint(q0) & 0xFFFFu;
  if (lo - 0x7FFAu <= 12u) q0 = __fdiv_rn(v, s);
  float r = rintf(bf16_round(q0));
  r = fminf(fmaxf(r, -128.0f), 127.0f);
  return (int)r;
}

// x_scale = bf16( bf16(max(amax, 1e-5)) / 127 )   (int8_linear.py:129)
__device__ __forceinline__ float act_scale(float amax_bf16) {
  float a = bf16_round(fmaxf(amax_bf16, 1e-5f));
  return bf16_round(__fdiv_rn(a, 127.0f));
}

// --- bit-reproducible fp32 exp / sigmoid / tanh ---------------------------
// exp(x) by Cody & Waite two-constant range reduction, x = k*ln2 + r with
// |r| <= ln2/2, and the degree-7 Taylor polynomial of e^r evaluated by Horner,
// then an exact scaling by 2^k.  Only IEEE fp32 operations with one rounding
// each (multiplies, adds, fused multiply-adds) are used, so the oracle replays
// it exactly.  Accuracy: within 2 ulp of exp on [-87, 88].
constexpr float kInvLn2 = 1.44269502f;
constexpr float kLn2Hi = 0.693145751953125f;   // 16 significant bits: k*kLn2Hi is exact
constexpr float kLn2Lo = 1.42860677e-06f;
constexpr float kExpC7 = 1.98412701e-04f;      // 1/7!
constexpr float kExpC6 = 1.38888892e-03f;      // 1/6!
constexpr float kExpC5 = 8.33333377e-03f;      // 1/5!
constexpr float kExpC4 = 4.16666679e-02f;      // 1/4!
constexpr float kExpC3 = 1.66666672e-01f;      // 1/3!

__device__ __forceinline__ float zib_expf(float x) {
  x = fminf(fmaxf(x, -87.0f), 88.0f);
  // k = rint(x / ln2) by the 1.5*2^23 shifter (round-half-even, |x / ln2| < 2^22);
  // its integer value is read from the shifted sum's low mantissa bits
  const float t = __fadd_rn(__fmul_rn(x, kInvLn2), 12582912.0f);
  const int ki = (int)__float_as_uint(t) - 0x4B400000;
  const float k = __fsub_rn(t, 12582912.0f);
  float r = __fmaf_rn(-k, kLn2Hi, x);
  r = __fmaf_rn(-k, kLn2Lo, r);
  float p = kExpC7;
  p = __fmaf_rn(p, r, kExpC6);
  p = __fmaf_rn(p, r, kExpC5);
  p = __fmaf_rn(p, r, kExpC4);
  p = __fmaf_rn(p, r, kExpC3);
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  // p * 2^k exactly: for x in [-87, 88], k is in [-126, 127] and p in [0.70, 1.42]
  // (p >= 1 when k = -126, since x >= -87 > -126 ln2), so the result is a normal
  // number and adding k to the exponent field equals ldexp
  return __uint_as_float(__float_as_uint(p) + ((uint32_t)ki << 23));
}

// exp(x) overflows fp32 for x above this (ln of the largest finite fp32, rounded down)
constexpr float kExpOverflow = 88.72283935546875f;

// sigmoid(g) = 1 / (1 + exp(-g)), the correctly rounded reciprocal; exactly 0 where
// exp(-g) overflows to inf in fp32 (the reference's fp32 sigmoid, swiglu.py:55)
__device__ __forceinline__ float zib_sigmoidf(float g) {
  const float s = __frcp_rn(__fadd_rn(1.0f, zib_expf(-g)));
  return -g > kExpOverflow ? 0.0f : s;
}

// tanh: odd Taylor polynomial (to x^11) for |x| < 0.25, else (1 - e^-2|x|) / (1 + e^-2|x|)
__device__ __forceinline__ float zib_tanhf(float x) {
  const float a = fabsf(x);
  float t;
  if (a < 0.25f) {
    const float x2 = __fmul_rn(a, a);
    float p = -8.86323552e-03f;                  // -1382/155925
    p = __fadd_rn(__fmul_rn(p, x2), 2.18694880e-02f);   // 62/2835
    p = __fadd_rn(__fmul_rn(p, x2), -5.39682545e-02f);  // -17/315
    p = __fadd_rn(__fmul_rn(p, x2), 1.33333340e-01f);   // 2/15
    p = __fadd_rn(__fmul_rn(p, x2), -3.33333343e-01f);  // -1/3
    t = __fadd_rn(a, __fmul_rn(__fmul_rn(p, x2), a));
  } else {
    const float e = zib_expf(__fmul_rn(-2.0f, a));
    t = __fdiv_rn(__fsub_rn(1.0f, e), __fadd_rn(1.0f, e));
  }
  return copysignf(t, x);
}

// rstd = 1 / sqrt(RN32(sum)/n + eps), IEEE fp32 ops
__device__ __forceinline__ float rstd_from_sum(double ss, int n, float eps) {
  float ms = __fdiv_rn((float)ss, (float)n);
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, eps)));
}

// --- 16-byte vector I/O --------------------------------------------------

struct alignas(16) bf16x8 { uint16_t h[8]; };

__device__ __forceinline__ void load_bf16x8(const void* p, float v[8]) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

__device__ __forceinline__ void load_bf16x8_nc(const void* p, float v[8]) {
  uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

// v[] must already hold bf16-exact values
__device__ __forceinline__ void store_bf16x8(void* p, const float v[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    w[i] = (__float_as_uint(v[2 * i]) >> 16) | (__float_as_uint(v[2 * i + 1]) & 0xFFFF0000u);
  }
  *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
}

__device__ __forceinline__ void store_i8x8(void* p, const int q[8]) {
  uint32_t a = (q[0] & 0xFF) | ((q[1] & 0xFF) << 8) | ((q[2] & 0xFF) << 16) | ((uint32_t)(q[3] & 0xFF) << 24);
  uint32_t b = (q[4] & 0xFF) | ((q[5] & 0xFF) << 8) | ((q[6] & 0xFF) << 16) | ((uint32_t)(q[7] & 0xFF) << 24);
  *reinterpret_cast<uint2*>(p) = make_uint2(a, b);
}

// --- cheap exact roundings --------------------------------------------------

// round a pair of fp32 values to bf16 (RNE), results as fp32
__device__ __forceinline__ void bf16_round2(float& a, float& b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  uint32_t w = *reinterpret_cast<uint32_t*>(&h);
  a = __uint_as_float(w << 16);
  b = __uint_as_float(w & 0xFFFF0000u);
}

// v[j] = mul_round_bf16(v[j], kHBf16) for 8 values: one RN multiply + packed
// rounding, with the exact-residual fix-up only when some lane of the warp has
// a product on a bf16 midpoint (every lane of the warp must call this)
__device__ __forceinline__ void had_round8(float v[8]) {
  float p[8];
  bool tie = false;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    p[j] = __fmul_rn(v[j], kHBf16);
    tie |= (__float_as_uint(p[j]) & 0xFFFFu) == 0x8000u;
  }
  if (__any_sync(0xFFFFFFFFu, tie)) {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = mul_round_bf16(v[j], kHBf16);
    return;
  }
#pragma unroll
  for (int j = 0; j < 8; j += 2) bf16_round2(p[j], p[j + 1]);
#pragma unroll
  for (int j = 0; j < 8; ++j) v[j] = p[j];
}

// --- Walsh-Hadamard transform over 128 (Sylvester order) ------------------
// A 128-group lives in 16 consecutive lanes x 8 values (lane bits 0..3 are
// index bits 3..6).  Index bits 0..2 are combined in-thread, bits 3..6 with
// xor shuffles.  All adds are exact for bf16-derived data in all practical
// cases (see the oracle's exactness notes).

__device__ __forceinline__ void fwht8(float v[8]) {
#pragma unroll
  for (int h = 1; h < 8; h <<= 1) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if ((i & h) == 0) {
        float a = v[i], b = v[i + h];
        v[i] = __fadd_rn(a, b);
        v[i + h] = __fsub_rn(a, b);
      }
    }
  }
}

__device__ __forceinline__ void fwht_cross16(float v[8], int lane) {
#pragma unroll
  for (int m = 1; m < 16; m <<= 1) {
    bool upper = (lane & m) != 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float o = __shfl_xor_sync(0xFFFFFFFFu, v[i], m);
      v[i] = upper ? __fsub_rn(o, v[i]) : __fadd_rn(v[i], o);
    }
  }
}

// --- block reductions -----------------------------------------------------

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  return v;
}

__device__ __forceinline__ double warp_sum_f64(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

// scratch must hold >= 32 entries; result broadcast to all threads
__device__ __forceinline__ float block_max(float v, float* scratch) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int nw = (blockDim.x + 31) >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) scratch[wid] = v;
  __syncthreads();
  float r = lane < nw ? scratch[lane] : 0.0f;
  return warp_max(r);
}

__device__ __forceinline__ double block_sum_f64(double v, double* scratch) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int nw = (blockDim.x + 31) >> 5;
  v = warp_sum_f64(v);
  __syncthreads();
  if (lane == 0) scratch[wid] = v;
  __syncthreads();
  double r = lane < nw ? scratch[lane] : 0.0;
  return warp_sum_f64(r);
}

}  // namespace zib
