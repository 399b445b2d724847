// Bandwidth-bound row kernels of the Z-Image W8A8 path (sm_100a).
//
// One CTA processes one row.  A row is split into 8-element chunks; chunk c
// is owned by thread (c mod blockDim), so a 128-element Hadamard group is
// held by 16 consecutive lanes (8 values each) and rotated with 3 in-thread
// butterfly stages plus 4 xor-shuffle stages.  Every kernel keeps the
// reference's bf16 rounding points; see zib_common.cuh.
#include "zib_async.cuh"
#include "rot_pack.cuh"

#include <stdio.h>

ZIB_DEFINE_ERROR_READER(zib_err_read_clear_rows)

namespace zib {

constexpr int kMaxCpt = 8;  // chunks per thread; 8 * 8 * 1024 = 65536 = MAX_FUSED_SIZE (kernels/utils.py:32)

// ---------------------------------------------------------------------------
// chunk I/O with a vector (16-byte) or scalar (ragged/misaligned) path
// ---------------------------------------------------------------------------
template <bool VEC>
__device__ __forceinline__ void ld_chunk(const uint16_t* row, int64_t c, int64_t n, float v[8]) {
  if (VEC) {
    load_bf16x8(row + c * 8, v);
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      int64_t e = c * 8 + j;
      v[j] = e < n ? bf16_bits_to_float(row[e]) : 0.0f;
    }
  }
}

template <bool VEC>
__device__ __forceinline__ void st_chunk(uint16_t* row, int64_t c, int64_t n, const float v[8]) {
  if (VEC) {
    store_bf16x8(row + c * 8, v);
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      int64_t e = c * 8 + j;
      if (e < n) row[e] = (uint16_t)(__float_as_uint(v[j]) >> 16);
    }
  }
}

template <bool VEC>
__device__ __forceinline__ void ld_w(const float* w, int64_t c, int64_t n, float v[8]) {
  if (VEC) {
    float4 a = __ldg(reinterpret_cast<const float4*>(w + c * 8));
    float4 b = __ldg(reinterpret_cast<const float4*>(w + c * 8 + 4));
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      int64_t e = c * 8 + j;
      v[j] = e < n ? w[e] : 0.0f;
    }
  }
}

// ---------------------------------------------------------------------------
// shared tail: rotate (optional) + amax + int8 quantisation of a row held in
// registers as bf16-exact floats.  All threads of the CTA must call it.
// ---------------------------------------------------------------------------
template <int CPT, bool HAD>
__device__ __forceinline__ void rotate_quant_row(float (&v)[CPT][8], int64_t row, int64_t nchunks,
                                                 int8_t* __restrict__ q, int64_t ldq,
                                                 uint16_t* __restrict__ sx, uint16_t* __restrict__ xrot,
                                                 float* red) {
  const int tid = threadIdx.x, lane = tid & 31;
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < CPT; ++i) {
    const int64_t c = tid + (int64_t)i * blockDim.x;
    if (HAD) {
      // Every lane of a half-warp takes part in the shuffles; a half-warp's
      // 16 chunks are all valid or all invalid because nchunks % 16 == 0.
      fwht8(v[i]);
      fwht_cross16(v[i], lane);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] = mul_round_bf16(v[i][j], kHBf16);
    }
    if (c < nchunks) {
#pragma unroll
      for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[i][j]));
    }
  }
  amax = block_max(amax, red);
  const float s = act_scale(amax);
  const float rcp = __fdiv_rn(1.0f, s);
#pragma unroll
  for (int i = 0; i < CPT; ++i) {
    const int64_t c = tid + (int64_t)i * blockDim.x;
    if (c < nchunks) {
      int qq[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) qq[j] = quant_i8(v[i][j], s, rcp);
      store_i8x8(q + row * ldq + c * 8, qq);
      if (xrot) store_bf16x8(xrot + row * ldq + c * 8, v[i]);
    }
  }
  if (tid == 0) sx[row] = float_to_bf16_bits(s);
}

// ---------------------------------------------------------------------------
// K2: activation rotation + quantisation (int8_linear.py:119-130)
// ---------------------------------------------------------------------------
template <int CPT, bool HAD>
__global__ void __launch_bounds__(1024) act_quant_kernel(const uint16_t* __restrict__ x, int64_t ldx,
                                                         int8_t* __restrict__ q, int64_t ldq,
                                                         uint16_t* __restrict__ sx, uint16_t* __restrict__ xrot,
                                                         int64_t n) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int64_t nchunks = n / 8;
  float v[CPT][8];
#pragma unroll
  for (int i = 0; i < CPT; ++i) {
    const int64_t c = threadIdx.x + (int64_t)i * blockDim.x;
    if (c < nchunks) load_bf16x8_nc(x + row * ldx + c * 8, v[i]);
    else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] = 0.0f;
    }
  }
  rotate_quant_row<CPT, HAD>(v, row, nchunks, q, ldq, sx, xrot, red);
}

// ---------------------------------------------------------------------------
// K5: RMSNorm (+ adaLN modulation) (+ rotation/quantisation)
//   MODE 0: y = rmsnorm(x)              (rms_norm.py:47-57)
//   MODE 1: y = rmsnorm(x) * (1 + s)    (+ shift)   (patching_comfyui.py:378)
//   MODE 2: MODE 1 then rotate + quantise (int8_linear.py:119-130)
// ---------------------------------------------------------------------------
template <int CPT, bool VEC, int MODE, bool HAD>
__global__ void __launch_bounds__(1024) rmsnorm_kernel(
    const uint16_t* __restrict__ x, int64_t ldx, const float* __restrict__ w,
    const uint16_t* __restrict__ scale, const uint16_t* __restrict__ shift, int64_t ld_mod,
    int64_t rows_per_batch, uint16_t* __restrict__ y, int64_t ldy,
    int8_t* __restrict__ q, int64_t ldq, uint16_t* __restrict__ sx, int64_t n, float eps) {
  __shared__ double redd[32];
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int64_t nchunks = (n + 7) / 8;
  const uint16_t* xr = x + row * ldx;
  float v[CPT][8];
  double ss = 0.0;
#pragma unroll
  for (int i = 0; i < CPT; ++i) {
    const int64_t c = threadIdx.x + (int64_t)i * blockDim.x;
    if (c < nchunks) {
      ld_chunk<VEC>(xr, c, n, v[i]);
      ss += (double)chunk_sumsq(v[i]);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] = 0.0f;
    }
  }
  ss = block_sum_f64(ss, redd);
  const float rstd = rstd_from_sum(ss, (int)n, eps);
  const int64_t b = row / rows_per_batch;
#pragma unroll
  for (int i = 0; i < CPT; ++i) {
    const int64_t c = threadIdx.x + (int64_t)i * blockDim.x;
    if (c < nchunks) {
      float wv[8];
      ld_w<VEC>(w, c, n, wv);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] = bf16_round(__fmul_rn(bf16_round(__fmul_rn(v[i][j], rstd)), wv[j]));
      if (MODE >= 1) {
        float sv[8];
        ld_chunk<VEC>(scale + b * ld_mod, c, n, sv);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] = bf16_round(__fmul_rn(v[i][j], bf16_round(__fadd_rn(1.0f, sv[j]))));
        if (shift) {
          ld_chunk<VEC>(shift + b * ld_mod, c, n, sv);
#pragma unroll
          for (int j = 0; j < 8; ++j) v[i][j] = bf16_round(__fadd_rn(v[i][j], sv[j]));
        }
      }
      if (MODE <= 1) st_chunk<VEC>(y + row * ldy, c, n, v[i]);
    }
  }
  if (MODE == 2) rotate_quant_row<CPT, HAD>(v, row, nchunks, q, ldq, sx, nullptr, red);
}

// ---------------------------------------------------------------------------
// K6: y = r + gate * rmsnorm(x)   (fused_norm_residual.py:58-73)
//   FUSE: then rmsnorm(y; w2) * (1 + s) (+ shift), rotate, quantise.
// ---------------------------------------------------------------------------
template <int CPT, bool VEC, bool FUSE, bool HAD>
__global__ void __launch_bounds__(1024) norm_gate_residual_kernel(
    const uint16_t* __restrict__ x, int64_t ldx, const uint16_t* __restrict__ r, int64_t ldr,
    const uint16_t* __restrict__ gate, int64_t ld_gate, int64_t rows_per_batch,
    const float* __restrict__ w, uint16_t* __restrict__ y, int64_t ldy,
    const float* __restrict__ w2, const uint16_t* __restrict__ scale, const uint16_t* __restrict__ shift,
    int64_t ld_mod, int8_t* __restrict__ q, int64_t ldq, uint16_t* __restrict__ sx,
    int64_t n, float eps, float eps2) {
  __shared__ double redd[32];
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int64_t nchunks = (n + 7) / 8;
  const int64_t b = row / rows_per_batch;
  float v[CPT][8];
  double ss = 0.0;
#pragma unroll
  for (int i = 0; i < CPT; ++i) {
    const int64_t c = threadIdx.x + (int64_t)i * blockDim.x;
    if (c < nchunks) {
      ld_chunk<VEC>(x + row * ldx, c, n, v[i]);
      ss += (double)chunk_sumsq(v[i]);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] = 0.0f;
    }
  }
  ss = block_sum_f64(ss, redd);
  const float rstd = rstd_from_sum(ss, (int)n, eps);
  double ss2 = 0.0;
#pragma unroll
  for (int i = 0; i < CPT; ++i) {
    const int64_t c = threadIdx.x + (int64_t)i * blockDim.x;
    if (c < nchunks) {
      float wv[8], gv[8], rv[8];
      ld_w<VEC>(w, c, n, wv);
      ld_chunk<VEC>(gate + b * ld_gate, c, n, gv);
      ld_chunk<VEC>(r + row * ldr, c, n, rv);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float xs = bf16_round(__fmul_rn(bf16_round(__fmul_rn(v[i][j], rstd)), wv[j]));
        v[i][j] = bf16_fma(gv[j], xs, rv[j]);  // RN_bf16(r + g * xs), one rounding
      }
      if (FUSE) ss2 += (double)chunk_sumsq(v[i]);
      st_chunk<VEC>(y + row * ldy, c, n, v[i]);
    }
  }
  if (FUSE) {
    ss2 = block_sum_f64(ss2, redd);
    const float rstd2 = rstd_from_sum(ss2, (int)n, eps2);
#pragma unroll
    for (int i = 0; i < CPT; ++i) {
      const int64_t c = threadIdx.x + (int64_t)i * blockDim.x;
      if (c < nchunks) {
        float wv[8], sv[8];
        ld_w<VEC>(w2, c, n, wv);
        ld_chunk<VEC>(scale + b * ld_mod, c, n, sv);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float z = bf16_round(__fmul_rn(bf16_round(__fmul_rn(v[i][j], rstd2)), wv[j]));
          v[i][j] = bf16_round(__fmul_rn(z, bf16_round(__fadd_rn(1.0f, sv[j]))));
        }
        if (shift) {
          ld_chunk<VEC>(shift + b * ld_mod, c, n, sv);
#pragma unroll
          for (int j = 0; j < 8; ++j) v[i][j] = bf16_round(__fadd_rn(v[i][j], sv[j]));
        }
      }
    }
    rotate_quant_row<CPT, HAD>(v, row, nchunks, q, ldq, sx, nullptr, red);
  }
}

// ---------------------------------------------------------------------------
// K4: SwiGLU  out = bf16(bf16(silu(g)) * u)   (swiglu.py:51-58)  (+ quant)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float silu_bf16(float g) {
  return bf16_round(__fmul_rn(g, zib_sigmoidf(g)));
}

template <int CPT, bool VEC, bool QUANT, bool HAD>
__global__ void __launch_bounds__(1024) swiglu_kernel(
    const uint16_t* __restrict__ g, int64_t ldg, const uint16_t* __restrict__ u, int64_t ldu,
    uint16_t* __restrict__ out, int64_t ldo, int8_t* __restrict__ q, int64_t ldq,
    uint16_t* __restrict__ sx, int64_t n) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int64_t nchunks = (n + 7) / 8;
  float v[CPT][8];
#pragma unroll
  for (int i = 0; i < CPT; ++i) {
    const int64_t c = threadIdx.x + (int64_t)i * blockDim.x;
    if (c < nchunks) {
      float gv[8], uv[8];
      ld_chunk<VEC>(g + row * ldg, c, n, gv);
      ld_chunk<VEC>(u + row * ldu, c, n, uv);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] = bf16_round(__fmul_rn(silu_bf16(gv[j]), uv[j]));
      if (!QUANT) st_chunk<VEC>(out + row * ldo, c, n, v[i]);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] = 0.0f;
    }
  }
  if (QUANT) rotate_quant_row<CPT, HAD>(v, row, nchunks, q, ldq, sx, nullptr, red);
}

// ---------------------------------------------------------------------------
// K3: per-head RMSNorm + interleaved RoPE, d = 128 (fused_qknorm_rope.py:85-151)
// One warp per token: its two half-warps take heads h0 + 2i (h0 = 0, 1), 16
// lanes per (token, head) row with 8 values (4 pairs) each, so that a warp's
// loads and stores cover two adjacent heads (512 contiguous bytes when the
// heads are packed) and the token's cos / sin, shared by all its heads, are
// loaded once instead of once per head.  RB rows per half-warp in flight.
// ---------------------------------------------------------------------------
template <bool NORM>
__global__ void __launch_bounds__(256) qknorm_rope_kernel(
    const uint16_t* __restrict__ x, int64_t x_sb, int64_t x_ss, int64_t x_sh,
    uint16_t* __restrict__ out, int64_t o_sb, int64_t o_ss, int64_t o_sh,
    const float* __restrict__ cosp, const float* __restrict__ sinp, int64_t cs_b,
    const float* __restrict__ w, int64_t S, int64_t H, int64_t tokens, float eps) {
  constexpr int RB = 5;
  const int lane = threadIdx.x & 31;
  const int sub = lane & 15;
  const int h0 = lane >> 4;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  float4 wa = make_float4(0.f, 0.f, 0.f, 0.f), wb = wa;
  if (NORM) {
    wa = __ldg(reinterpret_cast<const float4*>(w + sub * 8));
    wb = __ldg(reinterpret_cast<const float4*>(w + sub * 8 + 4));
  }
  for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < tokens; t += warps) {
    const int64_t b = t / S, s = t - b * S;
    const float4 c4 = __ldg(reinterpret_cast<const float4*>(cosp + b * cs_b + s * 64 + sub * 4));
    const float4 s4 = __ldg(reinterpret_cast<const float4*>(sinp + b * cs_b + s * 64 + sub * 4));
    const float cv[4] = {c4.x, c4.y, c4.z, c4.w};
    const float sv[4] = {s4.x, s4.y, s4.z, s4.w};
    const uint16_t* xt = x + b * x_sb + s * x_ss + sub * 8;
    uint16_t* ot = out + b * o_sb + s * o_ss + sub * 8;
    for (int64_t hb = h0; hb < H; hb += 2 * RB) {
      uint4 xv[RB];
#pragma unroll
      for (int r = 0; r < RB; ++r) {
        const int64_t h = hb + 2 * r;
        xv[r] = h < H ? *reinterpret_cast<const uint4*>(xt + h * x_sh) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int r = 0; r < RB; ++r) {
        uint4 v = xv[r];
        if (NORM) {
          // the row's canonical sum of squares (chunk sums added exactly across the 16 lanes),
          // then bf16(bf16(x * rstd) * w) two lanes per instruction
          double ss = px::sumsq_chunk(v);
#pragma unroll
          for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
          v = px::norm_w(v, rstd_from_sum(ss, 128, eps), wa, wb);
        }
        const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
        uint32_t o[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {  // pair rotation: fma(a, c, -(b s)), fma(b, c, a s)
          const float a = __uint_as_float(wv[k] << 16), bb = __uint_as_float(wv[k] & 0xFFFF0000u);
          o[k] = px::to_bf16x2(px::mk(__fmaf_rn(a, cv[k], -__fmul_rn(bb, sv[k])),
                                      __fmaf_rn(bb, cv[k], __fmul_rn(a, sv[k]))));
        }
        const int64_t h = hb + 2 * r;
        if (h < H) *reinterpret_cast<uint4*>(ot + h * o_sh) = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// adaLN (adaln_modulation.py:68-81; patching_comfyui.py:368-372)
// ---------------------------------------------------------------------------
__global__ void adaln_modulation_kernel(const uint16_t* __restrict__ raw, int64_t ldr,
                                        uint16_t* __restrict__ sm, uint16_t* __restrict__ gm,
                                        uint16_t* __restrict__ sp, uint16_t* __restrict__ gp,
                                        int64_t rows, int64_t dim) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * dim) return;
  const int64_t r = i / dim, c = i % dim;
  const uint16_t* rr = raw + r * ldr;
  sm[i] = float_to_bf16_bits(__fadd_rn(bf16_bits_to_float(rr[c]), 1.0f));
  gm[i] = float_to_bf16_bits(zib_tanhf(bf16_bits_to_float(rr[dim + c])));
  sp[i] = float_to_bf16_bits(__fadd_rn(bf16_bits_to_float(rr[2 * dim + c]), 1.0f));
  gp[i] = float_to_bf16_bits(zib_tanhf(bf16_bits_to_float(rr[3 * dim + c])));
}

__global__ void adaln_gates_kernel(const uint16_t* __restrict__ raw, int64_t ldr,
                                   uint16_t* __restrict__ gates, int64_t rows, int64_t dim) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * 2 * dim) return;
  const int64_t r = i / (2 * dim), k = (i / dim) % 2, c = i % dim;
  const uint16_t* rr = raw + r * ldr;
  gates[i] = float_to_bf16_bits(zib_tanhf(bf16_bits_to_float(rr[(2 * k + 1) * dim + c])));
}

// ---------------------------------------------------------------------------
// Weight prep (hadamard.py:47-75 + int8_linear.py:67-73), fp64 rotation
// ---------------------------------------------------------------------------
__device__ __forceinline__ void fwht8_f64(double v[8]) {
#pragma unroll
  for (int h = 1; h < 8; h <<= 1) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if ((i & h) == 0) {
        double a = v[i], b = v[i + h];
        v[i] = a + b;
        v[i + h] = a - b;
      }
    }
  }
}

__device__ __forceinline__ void fwht_cross16_f64(double v[8], int lane) {
#pragma unroll
  for (int m = 1; m < 16; m <<= 1) {
    bool upper = (lane & m) != 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      double o = __shfl_xor_sync(0xFFFFFFFFu, v[i], m);
      v[i] = upper ? o - v[i] : v[i] + o;
    }
  }
}

template <int CPT, bool HAD>
__global__ void __launch_bounds__(1024) weight_prep_kernel(
    const uint16_t* __restrict__ w, int64_t ldw, int8_t* __restrict__ wq, int64_t ldq,
    uint16_t* __restrict__ sw, float* __restrict__ sw32, float* __restrict__ wrot, int64_t ldr, int64_t n) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int64_t nchunks = n / 8;
  const int lane = threadIdx.x & 31;
  float v[CPT][8];
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < CPT; ++i) {
    const int64_t c = threadIdx.x + (int64_t)i * blockDim.x;
    float t[8];
    if (c < nchunks) load_bf16x8_nc(w + row * ldw + c * 8, t);
    else {
#pragma unroll
      for (int j = 0; j < 8; ++j) t[j] = 0.0f;
    }
    if (HAD) {
      double d[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) d[j] = (double)t[j];
      fwht8_f64(d);
      fwht_cross16_f64(d, lane);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] = __double2float_rn(d[j] * (double)kHFp32);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] = t[j];
    }
    if (c < nchunks) {
#pragma unroll
      for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[i][j]));
    }
  }
  amax = block_max(amax, red);
  const float s = __fdiv_rn(fmaxf(amax, 1e-5f), 127.0f);
#pragma unroll
  for (int i = 0; i < CPT; ++i) {
    const int64_t c = threadIdx.x + (int64_t)i * blockDim.x;
    if (c < nchunks) {
      int qq[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float r = rintf(__fdiv_rn(v[i][j], s));
        qq[j] = (int)fminf(fmaxf(r, -128.0f), 127.0f);
      }
      store_i8x8(wq + row * ldq + c * 8, qq);
      if (wrot) {
        float4* dst = reinterpret_cast<float4*>(wrot + row * ldr + c * 8);
        dst[0] = make_float4(v[i][0], v[i][1], v[i][2], v[i][3]);
        dst[1] = make_float4(v[i][4], v[i][5], v[i][6], v[i][7]);
      }
    }
  }
  if (threadIdx.x == 0) {
    sw[row] = float_to_bf16_bits(s);
    if (sw32) sw32[row] = s;
  }
}

// ---------------------------------------------------------------------------
// launch helpers
// ---------------------------------------------------------------------------
struct RowLaunch {
  int threads;
  int cpt;
};

// Picks threads (multiple of 32, <= 1024) and chunks per thread (1,2,4,8).
static inline bool row_launch(int64_t nchunks, RowLaunch* l) {
  int cpt = 1;
  while ((int64_t)cpt * 1024 < nchunks) cpt *= 2;
  if (cpt > kMaxCpt) return false;
  int64_t th = (nchunks + cpt - 1) / cpt;
  th = (th + 31) / 32 * 32;
  if (th < 32) th = 32;
  l->threads = (int)th;
  l->cpt = cpt;
  return true;
}

static inline bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

// ===========================================================================
// v3: persistent row pipeline, few warps per row
//
// A CTA of 32*W threads (W = 1, 2 or 4 warps) owns one row at a time and
// streams its rows (blockIdx.x, blockIdx.x + gridDim.x, ...) through a 2-3
// stage shared-memory ring filled by 1-D bulk async copies (thread 0 keeps the
// next rows in flight).  Each thread walks many 8-element chunks of the row
// (chunk c = tid + k*32W, so a 128-element Hadamard group always sits in 16
// consecutive lanes); intermediate results that must wait for a row statistic
// (RMS, absmax) are written back into the ring slot as bf16 and re-read in
// the next pass, so registers stay small while per-row costs (reductions,
// rstd/scale divisions, index math) are spread over 30-160 elements per thread.
// Same arithmetic as the v1 kernels.
// ===========================================================================
namespace pipe {

constexpr int kMaxStages = 3;

struct Ring {
  uint64_t* full;
  uint8_t* buf;
  uint32_t row_bytes;
  uint32_t stage_bytes;
  int stages;
};

__device__ __forceinline__ void ring_issue(const Ring& r, int slot, int64_t row, const uint16_t* in0, int64_t ld0,
                                           const uint16_t* in1, int64_t ld1) {
  uint64_t* bar = &r.full[slot];
  mbar_arrive_expect_tx(bar, r.stage_bytes);
  uint8_t* dst = r.buf + (size_t)slot * r.stage_bytes;
  bulk_g2s(dst, in0 + row * ld0, r.row_bytes, bar);
  if (in1) bulk_g2s(dst + r.row_bytes, in1 + row * ld1, r.row_bytes, bar);
}

struct Driver {
  Ring ring;
  int64_t first, stride, my_rows;
  const uint16_t *in0, *in1;
  int64_t ld0, ld1;
  int* abort_s;

  __device__ __forceinline__ int64_t row_of(int64_t i) const { return first + i * stride; }

  __device__ __forceinline__ void prologue() {
    if (threadIdx.x == 0)
      for (int j = 0; j < ring.stages - 1 && j < my_rows; ++j) ring_issue(ring, j, row_of(j), in0, ld0, in1, ld1);
  }

  // Issue row i+S-1 into the slot row i-1 used (every thread finished with it
  // before the trailing barrier of iteration i-1), then wait for row i.
  __device__ __forceinline__ bool wait(int64_t i) {
    const int S = ring.stages;
    const int slot = (int)(i % S);
    const uint32_t par = (uint32_t)((i / S) & 1);
    if (threadIdx.x == 0) {
      if (i + S - 1 < my_rows) ring_issue(ring, (int)((i + S - 1) % S), row_of(i + S - 1), in0, ld0, in1, ld1);
      if (!mbar_wait_bounded(&ring.full[slot], par, abort_s)) *abort_s = 1;
    }
    __syncthreads();
    if (*(volatile int*)abort_s) return false;
    mbar_try_wait(&ring.full[slot], par);  // completed: acquires the bulk-copy writes for this thread
    return true;
  }

  __device__ __forceinline__ void drain(int64_t i) {
    if (threadIdx.x != 0) return;
    const int S = ring.stages;
    for (int64_t k = i; k < my_rows && k < i + S; ++k)
      mbar_drain_wait(&ring.full[k % S], (uint32_t)((k / S) & 1));
  }

  __device__ __forceinline__ uint16_t* slot_ptr(int64_t i, int which) const {
    return reinterpret_cast<uint16_t*>(ring.buf + (size_t)(i % ring.stages) * ring.stage_bytes +
                                       which * ring.row_bytes);
  }
};

__device__ __forceinline__ Driver make_driver(uint8_t* smem, uint64_t* full, int* abort_s, int stages, int64_t n,
                                              int nin, int64_t rows, const uint16_t* in0, int64_t ld0,
                                              const uint16_t* in1, int64_t ld1) {
  Driver d;
  d.ring.full = full;
  d.ring.buf = smem;
  d.ring.row_bytes = (uint32_t)(n * 2);
  d.ring.stage_bytes = (uint32_t)(n * 2 * nin);
  d.ring.stages = stages;
  d.first = blockIdx.x;
  d.stride = gridDim.x;
  d.my_rows = d.first < rows ? (rows - d.first + d.stride - 1) / d.stride : 0;
  d.in0 = in0;
  d.in1 = in1;
  d.ld0 = ld0;
  d.ld1 = ld1;
  d.abort_s = abort_s;
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) mbar_init(&full[s], 1);
    *abort_s = 0;
    mbar_fence_init();
  }
  __syncthreads();
  return d;
}

// --- reductions over the CTA (W warps) -----------------------------------------

template <int W>
__device__ __forceinline__ float cta_max(float v, float* red) {
  v = warp_max(v);
  if (W == 1) return v;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float r = red[0];
#pragma unroll
  for (int k = 1; k < W; ++k) r = fmaxf(r, red[k]);
  __syncthreads();
  return r;
}

template <int W>
__device__ __forceinline__ double cta_sum(double v, double* red) {
  v = warp_sum_f64(v);
  if (W == 1) return v;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) red[wid] = v;
  __syncthreads();
  double r = red[0];
#pragma unroll
  for (int k = 1; k < W; ++k) r += red[k];
  __syncthreads();
  return r;
}

// --- cheap exact roundings ------------------------------------------------------

__device__ __forceinline__ void quant8(const float v[8], float s, float rcp, int q[8]) {
  float t[8];
  bool near = false;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    t[j] = __fmul_rn(v[j], rcp);
    near |= ((__float_as_uint(t[j]) & 0xFFFFu) - 0x7FFAu) <= 12u;
  }
  if (__any_sync(0xFFFFFFFFu, near)) {
#pragma unroll
    for (int j = 0; j < 8; ++j) q[j] = quant_i8(v[j], s, rcp);
    return;
  }
#pragma unroll
  for (int j = 0; j < 8; j += 2) bf16_round2(t[j], t[j + 1]);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    // round half to even and saturate to [-128, 127] in one conversion (low byte is stored)
    int i;
    asm("cvt.rni.sat.s8.f32 %0, %1;" : "=r"(i) : "f"(t[j]));
    q[j] = i;
  }
}

__device__ __forceinline__ void store_i8x8_prmt(void* p, const int q[8]) {
  uint32_t a = __byte_perm(__byte_perm(q[0], q[1], 0x0040), __byte_perm(q[2], q[3], 0x0040), 0x5410);
  uint32_t b = __byte_perm(__byte_perm(q[4], q[5], 0x0040), __byte_perm(q[6], q[7], 0x0040), 0x5410);
  *reinterpret_cast<uint2*>(p) = make_uint2(a, b);
}

__device__ __forceinline__ void fwht128(float v[8], int lane) {
  fwht8(v);
#pragma unroll
  for (int m = 1; m < 16; m <<= 1) {
    const float sg = (lane & m) ? -1.0f : 1.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float o = __shfl_xor_sync(0xFFFFFFFFu, v[i], m);
      v[i] = __fmaf_rn(sg, v[i], o);
    }
  }
}

// Rotate (optional) the bf16 chunk in place in shared memory and fold its absmax.
// Every lane of the warp must call this (shuffles), valid or not.
template <bool HAD>
__device__ __forceinline__ void rot_chunk_inplace(float v[8], bool valid, uint16_t* sp, float& amax, int lane) {
  if (HAD) {
    fwht128(v, lane);
    had_round8(v);
    if (valid) store_bf16x8(sp, v);
  }
  if (valid) {
#pragma unroll
    for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[j]));
  }
}

// Final pass: quantise the bf16 row held in shared memory.
template <int W>
__device__ __forceinline__ void quant_pass(const uint16_t* srow, int64_t nchunks, float amax, int64_t row,
                                           int8_t* __restrict__ q, int64_t ldq, uint16_t* __restrict__ sx,
                                           float* red) {
  amax = cta_max<W>(amax, red);
  const float s = act_scale(amax);
  const float rcp = __fdiv_rn(1.0f, s);
#pragma unroll 2
  for (int64_t c0 = 0; c0 < nchunks; c0 += 32 * W) {
    const int64_t c = c0 + threadIdx.x;
    const bool valid = c < nchunks;
    float v[8];
    if (valid) load_bf16x8(srow + c * 8, v);
    else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = 0.0f;
    }
    int qq[8];
    quant8(v, s, rcp, qq);
    if (valid) store_i8x8_prmt(q + row * ldq + c * 8, qq);
  }
  if (threadIdx.x == 0) sx[row] = float_to_bf16_bits(s);
}

// --- kernels -------------------------------------------------------------------

template <int W, bool HAD>
__global__ void __launch_bounds__(128) act_quant_pipe(const uint16_t* __restrict__ x, int64_t ldx,
                                                      int8_t* __restrict__ q, int64_t ldq,
                                                      uint16_t* __restrict__ sx, int64_t n, int64_t rows,
                                                      int stages) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t full[kMaxStages];
  __shared__ float red[4];
  __shared__ int abort_s;
  Driver d = make_driver(smem, full, &abort_s, stages, n, 1, rows, x, ldx, nullptr, 0);
  const int64_t nchunks = n / 8;
  const int lane = threadIdx.x & 31;
  d.prologue();
  for (int64_t i = 0; i < d.my_rows; ++i) {
    if (!d.wait(i)) { d.drain(i); return; }
    uint16_t* sr = d.slot_ptr(i, 0);
    float amax = 0.0f;
#pragma unroll 2
    for (int64_t c0 = 0; c0 < nchunks; c0 += 32 * W) {
      const int64_t c = c0 + threadIdx.x;
      const bool valid = c < nchunks;
      float v[8];
      if (valid) load_bf16x8(sr + c * 8, v);
      else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = 0.0f;
      }
      rot_chunk_inplace<HAD>(v, valid, sr + c * 8, amax, lane);
    }
    quant_pass<W>(sr, nchunks, amax, d.row_of(i), q, ldq, sx, red);
    __syncthreads();
  }
}

// MODE 0: rmsnorm -> bf16; 1: rmsnorm*(1+s)(+shift) -> bf16; 2: MODE 1 -> rotate/quant
template <int W, int MODE, bool HAD>
__global__ void __launch_bounds__(128) rmsnorm_pipe(const uint16_t* __restrict__ x, int64_t ldx,
                                                    const float* __restrict__ w, const uint16_t* __restrict__ scale,
                                                    const uint16_t* __restrict__ shift, int64_t ld_mod,
                                                    int64_t rows_per_batch, uint16_t* __restrict__ y, int64_t ldy,
                                                    int8_t* __restrict__ q, int64_t ldq, uint16_t* __restrict__ sx,
                                                    int64_t n, float eps, int64_t rows, int stages) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t full[kMaxStages];
  __shared__ double redd[4];
  __shared__ float red[4];
  __shared__ int abort_s;
  Driver d = make_driver(smem, full, &abort_s, stages, n, 1, rows, x, ldx, nullptr, 0);
  const int64_t nchunks = n / 8;
  const int lane = threadIdx.x & 31;
  d.prologue();
  for (int64_t i = 0; i < d.my_rows; ++i) {
    if (!d.wait(i)) { d.drain(i); return; }
    const int64_t row = d.row_of(i);
    uint16_t* sr = d.slot_ptr(i, 0);
    double ss = 0.0;
#pragma unroll 2
    for (int64_t c = threadIdx.x; c < nchunks; c += 32 * W) {
      float v[8];
      load_bf16x8(sr + c * 8, v);
      ss += (double)chunk_sumsq(v);
    }
    ss = cta_sum<W>(ss, redd);
    const float rstd = rstd_from_sum(ss, (int)n, eps);
    const int64_t b = row / rows_per_batch;
    float amax = 0.0f;
#pragma unroll 2
    for (int64_t c0 = 0; c0 < nchunks; c0 += 32 * W) {
      const int64_t c = c0 + threadIdx.x;
      const bool valid = c < nchunks;
      float v[8];
      if (valid) {
        float wv[8];
        load_bf16x8(sr + c * 8, v);
        ld_w<true>(w, c, n, wv);
#pragma unroll
        for (int j = 0; j < 8; j += 2) {
          float a0 = __fmul_rn(v[j], rstd), a1 = __fmul_rn(v[j + 1], rstd);
          bf16_round2(a0, a1);
          a0 = __fmul_rn(a0, wv[j]);
          a1 = __fmul_rn(a1, wv[j + 1]);
          bf16_round2(a0, a1);
          v[j] = a0;
          v[j + 1] = a1;
        }
        if (MODE >= 1) {
          float sv[8];
          load_bf16x8_nc(scale + b * ld_mod + c * 8, sv);
#pragma unroll
          for (int j = 0; j < 8; j += 2) {
            float m0 = __fadd_rn(1.0f, sv[j]), m1 = __fadd_rn(1.0f, sv[j + 1]);
            bf16_round2(m0, m1);
            float a0 = __fmul_rn(v[j], m0), a1 = __fmul_rn(v[j + 1], m1);
            bf16_round2(a0, a1);
            v[j] = a0;
            v[j + 1] = a1;
          }
          if (shift) {
            load_bf16x8_nc(shift + b * ld_mod + c * 8, sv);
#pragma unroll
            for (int j = 0; j < 8; j += 2) {
              float a0 = __fadd_rn(v[j], sv[j]), a1 = __fadd_rn(v[j + 1], sv[j + 1]);
              bf16_round2(a0, a1);
              v[j] = a0;
              v[j + 1] = a1;
            }
          }
        }
        if (MODE <= 1) store_bf16x8(y + row * ldy + c * 8, v);
        else if (!HAD) store_bf16x8(sr + c * 8, v);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = 0.0f;
      }
      if (MODE == 2) rot_chunk_inplace<HAD>(v, valid, sr + c * 8, amax, lane);
    }
    if (MODE == 2) quant_pass<W>(sr, nchunks, amax, row, q, ldq, sx, red);
    __syncthreads();
  }
}

// y = r + g*rmsnorm(x); FUSE: then rmsnorm(y;w2)*(1+s)(+shift) -> rotate/quant
template <int W, bool FUSE, bool HAD>
__global__ void __launch_bounds__(128) ngr_pipe(
    const uint16_t* __restrict__ x, int64_t ldx, const uint16_t* __restrict__ r, int64_t ldr,
    const uint16_t* __restrict__ gate, int64_t ld_gate, int64_t rows_per_batch, const float* __restrict__ w,
    uint16_t* __restrict__ y, int64_t ldy, const float* __restrict__ w2, const uint16_t* __restrict__ scale,
    const uint16_t* __restrict__ shift, int64_t ld_mod, int8_t* __restrict__ q, int64_t ldq,
    uint16_t* __restrict__ sx, int64_t n, float eps, float eps2, int64_t rows, int stages) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t full[kMaxStages];
  __shared__ double redd[4];
  __shared__ float red[4];
  __shared__ int abort_s;
  Driver d = make_driver(smem, full, &abort_s, stages, n, 1, rows, x, ldx, nullptr, 0);
  const int64_t nchunks = n / 8;
  const int lane = threadIdx.x & 31;
  d.prologue();
  for (int64_t i = 0; i < d.my_rows; ++i) {
    if (!d.wait(i)) { d.drain(i); return; }
    const int64_t row = d.row_of(i);
    uint16_t* sxr = d.slot_ptr(i, 0);  // x, later overwritten with y
    const uint16_t* rr = r + row * ldr;  // read once: straight from global
    const int64_t b = row / rows_per_batch;
    double ss = 0.0;
#pragma unroll 2
    for (int64_t c = threadIdx.x; c < nchunks; c += 32 * W) {
      float v[8];
      load_bf16x8(sxr + c * 8, v);
      ss += (double)chunk_sumsq(v);
    }
    ss = cta_sum<W>(ss, redd);
    const float rstd = rstd_from_sum(ss, (int)n, eps);
    double ss2 = 0.0;
#pragma unroll 2
    for (int64_t c = threadIdx.x; c < nchunks; c += 32 * W) {
      float v[8], wv[8], gv[8], rv[8];
      load_bf16x8(sxr + c * 8, v);
      load_bf16x8_nc(rr + c * 8, rv);
      ld_w<true>(w, c, n, wv);
      load_bf16x8_nc(gate + b * ld_gate + c * 8, gv);
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        float a0 = __fmul_rn(v[j], rstd), a1 = __fmul_rn(v[j + 1], rstd);
        bf16_round2(a0, a1);
        a0 = __fmul_rn(a0, wv[j]);
        a1 = __fmul_rn(a1, wv[j + 1]);
        bf16_round2(a0, a1);
        a0 = bf16_fma(gv[j], a0, rv[j]);  // RN_bf16(r + g * xs), one rounding
        a1 = bf16_fma(gv[j + 1], a1, rv[j + 1]);
        v[j] = a0;
        v[j + 1] = a1;
      }
      if (FUSE) ss2 += (double)chunk_sumsq(v);
      store_bf16x8(y + row * ldy + c * 8, v);
      if (FUSE) store_bf16x8(sxr + c * 8, v);
    }
    if (FUSE) {
      ss2 = cta_sum<W>(ss2, redd);
      const float rstd2 = rstd_from_sum(ss2, (int)n, eps2);
      float amax = 0.0f;
  #pragma unroll 2
    for (int64_t c0 = 0; c0 < nchunks; c0 += 32 * W) {
        const int64_t c = c0 + threadIdx.x;
        const bool valid = c < nchunks;
        float v[8];
        if (valid) {
          float wv[8], sv[8];
          load_bf16x8(sxr + c * 8, v);
          ld_w<true>(w2, c, n, wv);
          load_bf16x8_nc(scale + b * ld_mod + c * 8, sv);
#pragma unroll
          for (int j = 0; j < 8; j += 2) {
            float a0 = __fmul_rn(v[j], rstd2), a1 = __fmul_rn(v[j + 1], rstd2);
            bf16_round2(a0, a1);
            a0 = __fmul_rn(a0, wv[j]);
            a1 = __fmul_rn(a1, wv[j + 1]);
            bf16_round2(a0, a1);
            float m0 = __fadd_rn(1.0f, sv[j]), m1 = __fadd_rn(1.0f, sv[j + 1]);
            bf16_round2(m0, m1);
            a0 = __fmul_rn(a0, m0);
            a1 = __fmul_rn(a1, m1);
            bf16_round2(a0, a1);
            v[j] = a0;
            v[j + 1] = a1;
          }
          if (shift) {
            load_bf16x8_nc(shift + b * ld_mod + c * 8, sv);
#pragma unroll
            for (int j = 0; j < 8; j += 2) {
              float a0 = __fadd_rn(v[j], sv[j]), a1 = __fadd_rn(v[j + 1], sv[j + 1]);
              bf16_round2(a0, a1);
              v[j] = a0;
              v[j + 1] = a1;
            }
          }
          if (!HAD) store_bf16x8(sxr + c * 8, v);
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) v[j] = 0.0f;
        }
        rot_chunk_inplace<HAD>(v, valid, sxr + c * 8, amax, lane);
      }
      quant_pass<W>(sxr, nchunks, amax, row, q, ldq, sx, red);
    }
    __syncthreads();
  }
}

// out = bf16(bf16(silu(g)) * u); QUANT: rotate/quant instead of storing out
template <int W, bool QUANT, bool HAD>
__global__ void __launch_bounds__(128) swiglu_pipe(const uint16_t* __restrict__ g, int64_t ldg,
                                                   const uint16_t* __restrict__ u, int64_t ldu,
                                                   uint16_t* __restrict__ out, int64_t ldo, int8_t* __restrict__ q,
                                                   int64_t ldq, uint16_t* __restrict__ sx, int64_t n, int64_t rows,
                                                   int stages) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t full[kMaxStages];
  __shared__ float red[4];
  __shared__ int abort_s;
  Driver d = make_driver(smem, full, &abort_s, stages, n, 1, rows, g, ldg, nullptr, 0);
  const int64_t nchunks = n / 8;
  const int lane = threadIdx.x & 31;
  d.prologue();
  for (int64_t i = 0; i < d.my_rows; ++i) {
    if (!d.wait(i)) { d.drain(i); return; }
    const int64_t row = d.row_of(i);
    uint16_t* sg = d.slot_ptr(i, 0);
    const uint16_t* su = u + row * ldu;  // read once: straight from global
    float amax = 0.0f;
#pragma unroll 2
    for (int64_t c0 = 0; c0 < nchunks; c0 += 32 * W) {
      const int64_t c = c0 + threadIdx.x;
      const bool valid = c < nchunks;
      float v[8];
      if (valid) {
        float gv[8], uv[8];
        load_bf16x8(sg + c * 8, gv);
        load_bf16x8_nc(su + c * 8, uv);
#pragma unroll
        for (int j = 0; j < 8; j += 2) {
          float a0 = __fmul_rn(gv[j], zib_sigmoidf(gv[j])), a1 = __fmul_rn(gv[j + 1], zib_sigmoidf(gv[j + 1]));
          bf16_round2(a0, a1);
          a0 = __fmul_rn(a0, uv[j]);
          a1 = __fmul_rn(a1, uv[j + 1]);
          bf16_round2(a0, a1);
          v[j] = a0;
          v[j + 1] = a1;
        }
        if (!QUANT) store_bf16x8(out + row * ldo + c * 8, v);
        else if (!HAD) store_bf16x8(sg + c * 8, v);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = 0.0f;
      }
      if (QUANT) rot_chunk_inplace<HAD>(v, valid, sg + c * 8, amax, lane);
    }
    if (QUANT) quant_pass<W>(sg, nchunks, amax, row, q, ldq, sx, red);
    __syncthreads();
  }
}

// --- host launch helpers ---------------------------------------------------------

struct PipeCfg {
  int threads, warps, stages, grid;
  size_t smem;
};

static int num_sms() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

// Warps per row (CTA size 32*W): 4 keeps ~40 warps per SM at the Z-Image row lengths.
static inline int pipe_warps(int64_t) { return 4; }

template <class K>
static bool pipe_cfg(K kernel, int64_t n, int nin, int64_t rows, int warps, PipeCfg* c) {
  c->warps = warps;
  c->threads = 32 * warps;
  const size_t stage = (size_t)n * 2 * nin;
  c->stages = stage <= 16 * 1024 ? 3 : 2;
  c->smem = stage * c->stages;
  if (c->smem > 160 * 1024) return false;
  if (c->smem > 48 * 1024 &&
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)c->smem) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, c->threads, c->smem) != cudaSuccess ||
      per_sm < 1) {
    cudaGetLastError();
    return false;
  }
  int64_t g = (int64_t)per_sm * num_sms();
  c->grid = (int)(g < rows ? g : rows);
  return true;
}

}  // namespace pipe

#include "rows_warp.cuh"

}  // namespace zib

using namespace zib;

#define ZIB_DISPATCH_CPT(cpt, ...)              \
  switch (cpt) {                                \
    case 1: { constexpr int CPT = 1; __VA_ARGS__; } break; \
    case 2: { constexpr int CPT = 2; __VA_ARGS__; } break; \
    case 4: { constexpr int CPT = 4; __VA_ARGS__; } break; \
    default: { constexpr int CPT = 8; __VA_ARGS__; } break; \
  }


#define ZIB_DISPATCH_W(warps, ...)                                  \
  switch (warps) {                                                 \
    case 1: { constexpr int W = 1; __VA_ARGS__; } break;            \
    case 2: { constexpr int W = 2; __VA_ARGS__; } break;            \
    default: { constexpr int W = 4; __VA_ARGS__; } break;           \
  }

#define ZIB_PIPE_TRY(KERNEL, NIN, ROWS, N, ...)                                                 \
  do {                                                                                         \
    pipe::PipeCfg pc_;                                                                         \
    if (pipe::pipe_cfg(KERNEL, (N), (NIN), (ROWS), W, &pc_)) {                                  \
      KERNEL<<<pc_.grid, pc_.threads, pc_.smem, st>>>(__VA_ARGS__, (ROWS), pc_.stages);        \
      launched = true;                                                                         \
    }                                                                                          \
  } while (0)

#define ZIB_DISPATCH_BOOL(flag, NAME, ...)      \
  if (flag) { constexpr bool NAME = true; __VA_ARGS__; } \
  else { constexpr bool NAME = false; __VA_ARGS__; }

extern "C" int zib_act_quant(const void* x, int64_t ldx, void* q, int64_t ldq, void* sx,
                             void* x_rot, int64_t M, int64_t K, int hadamard, void* stream) {
  ZIB_HOST_CHECK(x && q && sx, ZIB_ERR_INVALID_ARG, "act_quant: null pointer");
  ZIB_HOST_CHECK(M >= 0 && K > 0, ZIB_ERR_INVALID_ARG, "act_quant: bad shape M=%lld K=%lld", (long long)M, (long long)K);
  ZIB_HOST_CHECK(K % 8 == 0, ZIB_ERR_INVALID_ARG, "act_quant: K=%lld must be a multiple of 8", (long long)K);
  ZIB_HOST_CHECK(!hadamard || K % kGroup == 0, ZIB_ERR_INVALID_ARG,
                 "act_quant: features %lld not divisible by group_size %d", (long long)K, kGroup);
  ZIB_HOST_CHECK(ldx >= K && ldq >= K && ldx % 8 == 0 && ldq % 8 == 0 && aligned16(x) && aligned16(q) &&
                     (!x_rot || aligned16(x_rot)),
                 ZIB_ERR_ALIGNMENT, "act_quant: rows must be 16-byte aligned");
  if (M == 0) return ZIB_OK;
  RowLaunch l;
  ZIB_HOST_CHECK(row_launch(K / 8, &l), ZIB_ERR_TOO_LARGE, "act_quant: K=%lld exceeds 65536", (long long)K);
  cudaStream_t st = (cudaStream_t)stream;
  bool launched = false;
  int rg_R = 0, rg_cpl = 0;
  if (wr::rg_shape(K, &rg_R, &rg_cpl)) {
    auto go = [&](auto k, int R) {
      k<<<wr::grid_rg(k, 32 * wr::warps_of(R), wr::warps_of(R) / R, M), 32 * wr::warps_of(R), 0, st>>>(
          (const uint16_t*)x, ldx, (int8_t*)q, ldq, (uint16_t*)sx, (uint16_t*)x_rot, M);
    };
    if (rg_R == 3) hadamard ? go(wr::act_quant_rg<3, 5, true>, 3) : go(wr::act_quant_rg<3, 5, false>, 3);
    else hadamard ? go(wr::act_quant_rg<4, 10, true>, 4) : go(wr::act_quant_rg<4, 10, false>, 4);
    launched = true;
  }
  if (!launched)
  launched = wr::dispatch(K, [&](auto Rc, int cpl) {
    constexpr int R = decltype(Rc)::value;
    auto k = hadamard ? wr::act_quant_wr<R, true> : wr::act_quant_wr<R, false>;
    wr::set_smem(k, wr::smem_for(R, cpl, 1));
    k<<<wr::grid_for(k, R, cpl, 1, M), 32 * wr::warps_of(R), wr::smem_for(R, cpl, 1), st>>>(
        (const uint16_t*)x, ldx, (int8_t*)q, ldq, (uint16_t*)sx, (uint16_t*)x_rot, cpl, M);
  });
  if (!launched && !x_rot)
    ZIB_DISPATCH_W(pipe::pipe_warps(K), ZIB_DISPATCH_BOOL(hadamard, HAD,
        ZIB_PIPE_TRY((pipe::act_quant_pipe<W, HAD>), 1, M, K,
                     (const uint16_t*)x, ldx, (int8_t*)q, ldq, (uint16_t*)sx, K)));
  if (!launched)  // other widths, or the rotated copy requested (direct-load kernel)
    ZIB_DISPATCH_CPT(l.cpt, ZIB_DISPATCH_BOOL(hadamard, HAD,
        act_quant_kernel<CPT, HAD><<<(unsigned)M, l.threads, 0, st>>>(
            (const uint16_t*)x, ldx, (int8_t*)q, ldq, (uint16_t*)sx, (uint16_t*)x_rot, K)));
  return zib_check_launch("act_quant");
}

extern "C" int zib_rms_norm(const void* x, int64_t ldx, const float* w, void* y, int64_t ldy,
                            int64_t rows, int64_t n, float eps, void* stream) {
  ZIB_HOST_CHECK(x && w && y, ZIB_ERR_INVALID_ARG, "rms_norm: null pointer");
  ZIB_HOST_CHECK(rows >= 0 && n > 0 && ldx >= n && ldy >= n, ZIB_ERR_INVALID_ARG, "rms_norm: bad shape");
  if (rows == 0) return ZIB_OK;
  RowLaunch l;
  ZIB_HOST_CHECK(row_launch((n + 7) / 8, &l), ZIB_ERR_TOO_LARGE,
                 "Cannot launch kernel since n = %lld exceeds the maximum fused size 65536.", (long long)n);
  const bool vec = n % 8 == 0 && ldx % 8 == 0 && ldy % 8 == 0 && aligned16(x) && aligned16(y) && aligned16(w);
  cudaStream_t st = (cudaStream_t)stream;
  bool launched = false;
  if (vec)
    launched = wr::dispatch(n, [&](auto Rc, int cpl) {
      constexpr int R = decltype(Rc)::value;
      auto k = wr::rmsnorm_wr<R, 0, false>;
      wr::set_smem(k, wr::smem_for(R, cpl, 1));
      k<<<wr::grid_for(k, R, cpl, 1, rows), 32 * wr::warps_of(R), wr::smem_for(R, cpl, 1), st>>>(
          (const uint16_t*)x, ldx, w, nullptr, nullptr, 0, 1, (uint16_t*)y, ldy, nullptr, 0, nullptr, n, eps, cpl,
          rows);
    });
  if (vec && !launched)
    ZIB_DISPATCH_W(pipe::pipe_warps(n), ZIB_PIPE_TRY((pipe::rmsnorm_pipe<W, 0, false>), 1, rows, n,
        (const uint16_t*)x, ldx, w, nullptr, nullptr, 0, 1, (uint16_t*)y, ldy, nullptr, 0, nullptr, n, eps));
  if (!launched)
    ZIB_DISPATCH_CPT(l.cpt, ZIB_DISPATCH_BOOL(vec, VEC,
        rmsnorm_kernel<CPT, VEC, 0, false><<<(unsigned)rows, l.threads, 0, st>>>(
            (const uint16_t*)x, ldx, w, nullptr, nullptr, 0, 1, (uint16_t*)y, ldy, nullptr, 0, nullptr, n, eps)));
  return zib_check_launch("rms_norm");
}

extern "C" int zib_rmsnorm_mod(const void* x, int64_t ldx, const float* w, const void* scale,
                               const void* shift, int64_t ld_mod, int64_t rows_per_batch,
                               void* y, int64_t ldy, int64_t rows, int64_t n, float eps, void* stream) {
  ZIB_HOST_CHECK(x && w && scale && y, ZIB_ERR_INVALID_ARG, "rmsnorm_mod: null pointer");
  ZIB_HOST_CHECK(rows >= 0 && n > 0 && ldx >= n && ldy >= n && ld_mod >= 0 && rows_per_batch > 0,
                 ZIB_ERR_INVALID_ARG, "rmsnorm_mod: bad shape");
  if (rows == 0) return ZIB_OK;
  RowLaunch l;
  ZIB_HOST_CHECK(row_launch((n + 7) / 8, &l), ZIB_ERR_TOO_LARGE, "rmsnorm_mod: n=%lld too large", (long long)n);
  const bool vec = n % 8 == 0 && ldx % 8 == 0 && ldy % 8 == 0 && ld_mod % 8 == 0 && aligned16(x) &&
                   aligned16(y) && aligned16(w) && aligned16(scale) && (!shift || aligned16(shift));
  cudaStream_t st = (cudaStream_t)stream;
  bool launched = false;
  if (vec)
    launched = wr::dispatch(n, [&](auto Rc, int cpl) {
      constexpr int R = decltype(Rc)::value;
      auto k = wr::rmsnorm_wr<R, 1, false>;
      wr::set_smem(k, wr::smem_for(R, cpl, 1));
      k<<<wr::grid_for(k, R, cpl, 1, rows), 32 * wr::warps_of(R), wr::smem_for(R, cpl, 1), st>>>(
          (const uint16_t*)x, ldx, w, (const uint16_t*)scale, (const uint16_t*)shift, ld_mod, rows_per_batch,
          (uint16_t*)y, ldy, nullptr, 0, nullptr, n, eps, cpl, rows);
    });
  if (vec && !launched)
    ZIB_DISPATCH_W(pipe::pipe_warps(n), ZIB_PIPE_TRY((pipe::rmsnorm_pipe<W, 1, false>), 1, rows, n,
        (const uint16_t*)x, ldx, w, (const uint16_t*)scale, (const uint16_t*)shift, ld_mod, rows_per_batch,
        (uint16_t*)y, ldy, nullptr, 0, nullptr, n, eps));
  if (!launched)
    ZIB_DISPATCH_CPT(l.cpt, ZIB_DISPATCH_BOOL(vec, VEC,
        rmsnorm_kernel<CPT, VEC, 1, false><<<(unsigned)rows, l.threads, 0, st>>>(
            (const uint16_t*)x, ldx, w, (const uint16_t*)scale, (const uint16_t*)shift, ld_mod, rows_per_batch,
            (uint16_t*)y, ldy, nullptr, 0, nullptr, n, eps)));
  return zib_check_launch("rmsnorm_mod");
}

extern "C" int zib_rmsnorm_mod_quant(const void* x, int64_t ldx, const float* w, const void* scale,
                                     const void* shift, int64_t ld_mod, int64_t rows_per_batch,
                                     void* q, int64_t ldq, void* sx, int64_t rows, int64_t n,
                                     float eps, int hadamard, void* stream) {
  ZIB_HOST_CHECK(x && w && scale && q && sx, ZIB_ERR_INVALID_ARG, "rmsnorm_mod_quant: null pointer");
  ZIB_HOST_CHECK(rows >= 0 && n > 0 && n % 8 == 0 && (!hadamard || n % kGroup == 0) && rows_per_batch > 0,
                 ZIB_ERR_INVALID_ARG, "rmsnorm_mod_quant: bad shape n=%lld", (long long)n);
  ZIB_HOST_CHECK(ldx % 8 == 0 && ldq % 8 == 0 && ld_mod % 8 == 0 && aligned16(x) && aligned16(q) &&
                     aligned16(w) && aligned16(scale) && (!shift || aligned16(shift)),
                 ZIB_ERR_ALIGNMENT, "rmsnorm_mod_quant: misaligned operand");
  if (rows == 0) return ZIB_OK;
  RowLaunch l;
  ZIB_HOST_CHECK(row_launch(n / 8, &l), ZIB_ERR_TOO_LARGE, "rmsnorm_mod_quant: n too large");
  cudaStream_t st = (cudaStream_t)stream;
  bool launched = false;
  if (n == 3840) {  // the register-resident kernel (teams of three warps, five chunks per lane)
    auto k = hadamard ? wr::rmsnorm_mod_quant_rg<3, 5, true> : wr::rmsnorm_mod_quant_rg<3, 5, false>;
    k<<<wr::grid_rg(k, 96, 1, rows), 96, 0, st>>>((const uint16_t*)x, ldx, w, (const uint16_t*)scale,
                                                  (const uint16_t*)shift, ld_mod, rows_per_batch, (int8_t*)q,
                                                  ldq, (uint16_t*)sx, n, eps, rows);
    launched = true;
  }
  if (!launched)
  launched = wr::dispatch(n, [&](auto Rc, int cpl) {
    constexpr int R = decltype(Rc)::value;
    auto k = hadamard ? wr::rmsnorm_wr<R, 2, true> : wr::rmsnorm_wr<R, 2, false>;
    wr::set_smem(k, wr::smem_for(R, cpl, 1));
    k<<<wr::grid_for(k, R, cpl, 1, rows), 32 * wr::warps_of(R), wr::smem_for(R, cpl, 1), st>>>(
        (const uint16_t*)x, ldx, w, (const uint16_t*)scale, (const uint16_t*)shift, ld_mod, rows_per_batch,
        nullptr, 0, (int8_t*)q, ldq, (uint16_t*)sx, n, eps, cpl, rows);
  });
  if (!launched)
  ZIB_DISPATCH_W(pipe::pipe_warps(n), ZIB_DISPATCH_BOOL(hadamard, HAD,
      ZIB_PIPE_TRY((pipe::rmsnorm_pipe<W, 2, HAD>), 1, rows, n,
          (const uint16_t*)x, ldx, w, (const uint16_t*)scale, (const uint16_t*)shift, ld_mod, rows_per_batch,
          nullptr, 0, (int8_t*)q, ldq, (uint16_t*)sx, n, eps)));
  if (!launched)
    ZIB_DISPATCH_CPT(l.cpt, ZIB_DISPATCH_BOOL(hadamard, HAD,
        rmsnorm_kernel<CPT, true, 2, HAD><<<(unsigned)rows, l.threads, 0, st>>>(
            (const uint16_t*)x, ldx, w, (const uint16_t*)scale, (const uint16_t*)shift, ld_mod, rows_per_batch,
            nullptr, 0, (int8_t*)q, ldq, (uint16_t*)sx, n, eps)));
  return zib_check_launch("rmsnorm_mod_quant");
}

extern "C" int zib_norm_gate_residual(const void* x, int64_t ldx, const void* r, int64_t ldr,
                                      const void* gate, int64_t ld_gate, int64_t rows_per_batch,
                                      const float* w, void* y, int64_t ldy, int64_t rows, int64_t n,
                                      float eps, void* stream) {
  ZIB_HOST_CHECK(x && r && gate && w && y, ZIB_ERR_INVALID_ARG, "norm_gate_residual: null pointer");
  ZIB_HOST_CHECK(rows >= 0 && n > 0 && rows_per_batch > 0 && ldx >= n && ldr >= n && ldy >= n,
                 ZIB_ERR_INVALID_ARG, "norm_gate_residual: bad shape");
  if (rows == 0) return ZIB_OK;
  RowLaunch l;
  ZIB_HOST_CHECK(row_launch((n + 7) / 8, &l), ZIB_ERR_TOO_LARGE, "norm_gate_residual: n too large");
  const bool vec = n % 8 == 0 && ldx % 8 == 0 && ldr % 8 == 0 && ldy % 8 == 0 && ld_gate % 8 == 0 &&
                   aligned16(x) && aligned16(r) && aligned16(y) && aligned16(gate) && aligned16(w);
  cudaStream_t st = (cudaStream_t)stream;
  bool launched = false;
  if (vec)
    launched = wr::dispatch<true>(n, [&](auto Rc, int cpl) {
      constexpr int R = decltype(Rc)::value;
      constexpr int nb = wr::ngr_buffers(R);
      auto k = wr::ngr_wr<R, false, false>;
      wr::set_smem(k, wr::smem_for(R, cpl, nb));
      k<<<wr::grid_for(k, R, cpl, nb, rows), 32 * wr::warps_of(R), wr::smem_for(R, cpl, nb), st>>>(
          (const uint16_t*)x, ldx, (const uint16_t*)r, ldr, (const uint16_t*)gate, ld_gate, rows_per_batch, w,
          (uint16_t*)y, ldy, nullptr, nullptr, nullptr, 0, nullptr, 0, nullptr, n, eps, eps, cpl, rows);
    });
  if (vec && !launched)
    ZIB_DISPATCH_W(pipe::pipe_warps(n), ZIB_PIPE_TRY((pipe::ngr_pipe<W, false, false>), 1, rows, n,
        (const uint16_t*)x, ldx, (const uint16_t*)r, ldr, (const uint16_t*)gate, ld_gate, rows_per_batch,
        w, (uint16_t*)y, ldy, nullptr, nullptr, nullptr, 0, nullptr, 0, nullptr, n, eps, eps));
  if (!launched)
    ZIB_DISPATCH_CPT(l.cpt, ZIB_DISPATCH_BOOL(vec, VEC,
        norm_gate_residual_kernel<CPT, VEC, false, false><<<(unsigned)rows, l.threads, 0, st>>>(
            (const uint16_t*)x, ldx, (const uint16_t*)r, ldr, (const uint16_t*)gate, ld_gate, rows_per_batch,
            w, (uint16_t*)y, ldy, nullptr, nullptr, nullptr, 0, nullptr, 0, nullptr, n, eps, eps)));
  return zib_check_launch("norm_gate_residual");
}

extern "C" int zib_norm_gate_residual_mod_quant(const void* x, int64_t ldx, const void* r, int64_t ldr,
                                                const void* gate, int64_t ld_gate, int64_t rows_per_batch,
                                                const float* w, void* y, int64_t ldy,
                                                const float* w2, const void* scale, const void* shift,
                                                int64_t ld_mod, void* q, int64_t ldq, void* sx,
                                                int64_t rows, int64_t n, float eps, float eps2,
                                                int hadamard, void* stream) {
  ZIB_HOST_CHECK(x && r && gate && w && y && w2 && scale && q && sx, ZIB_ERR_INVALID_ARG,
                 "norm_gate_residual_mod_quant: null pointer");
  ZIB_HOST_CHECK(rows >= 0 && n > 0 && n % 8 == 0 && (!hadamard || n % kGroup == 0) && rows_per_batch > 0,
                 ZIB_ERR_INVALID_ARG, "norm_gate_residual_mod_quant: bad shape");
  ZIB_HOST_CHECK(ldx % 8 == 0 && ldr % 8 == 0 && ldy % 8 == 0 && ld_gate % 8 == 0 && ld_mod % 8 == 0 &&
                     ldq % 8 == 0 && aligned16(x) && aligned16(r) && aligned16(y) && aligned16(gate) &&
                     aligned16(w) && aligned16(w2) && aligned16(scale) && aligned16(q) && (!shift || aligned16(shift)),
                 ZIB_ERR_ALIGNMENT, "norm_gate_residual_mod_quant: misaligned operand");
  if (rows == 0) return ZIB_OK;
  RowLaunch l;
  ZIB_HOST_CHECK(row_launch(n / 8, &l), ZIB_ERR_TOO_LARGE, "norm_gate_residual_mod_quant: n too large");
  cudaStream_t st = (cudaStream_t)stream;
  bool launched = false;
  if (n == 3840) {  // the register-resident kernel (teams of three warps, five chunks per lane)
    auto k = hadamard ? wr::ngr_rg<5, true, false> : wr::ngr_rg<5, false, false>;
    k<<<wr::grid_rg(k, 96, 1, rows), 96, 0, st>>>(
        (const uint16_t*)x, ldx, (const uint16_t*)r, ldr, (const uint16_t*)gate, ld_gate, rows_per_batch, w,
        (uint16_t*)y, ldy, w2, (const uint16_t*)scale, (const uint16_t*)shift, ld_mod, (int8_t*)q, ldq,
        (uint16_t*)sx, n, eps, eps2, rows);
    launched = true;
  }
  if (!launched)
  launched = wr::dispatch<true>(n, [&](auto Rc, int cpl) {
    constexpr int R = decltype(Rc)::value;
    constexpr int nb = wr::ngr_buffers(R);
    auto k = hadamard ? wr::ngr_wr<R, true, true> : wr::ngr_wr<R, true, false>;
    wr::set_smem(k, wr::smem_for(R, cpl, nb));
    k<<<wr::grid_for(k, R, cpl, nb, rows), 32 * wr::warps_of(R), wr::smem_for(R, cpl, nb), st>>>(
        (const uint16_t*)x, ldx, (const uint16_t*)r, ldr, (const uint16_t*)gate, ld_gate, rows_per_batch, w,
        (uint16_t*)y, ldy, w2, (const uint16_t*)scale, (const uint16_t*)shift, ld_mod, (int8_t*)q, ldq,
        (uint16_t*)sx, n, eps, eps2, cpl, rows);
  });
  if (!launched)
  ZIB_DISPATCH_W(pipe::pipe_warps(n), ZIB_DISPATCH_BOOL(hadamard, HAD,
      ZIB_PIPE_TRY((pipe::ngr_pipe<W, true, HAD>), 1, rows, n,
          (const uint16_t*)x, ldx, (const uint16_t*)r, ldr, (const uint16_t*)gate, ld_gate, rows_per_batch,
          w, (uint16_t*)y, ldy, w2, (const uint16_t*)scale, (const uint16_t*)shift, ld_mod, (int8_t*)q, ldq,
          (uint16_t*)sx, n, eps, eps2)));
  if (!launched)
    ZIB_DISPATCH_CPT(l.cpt, ZIB_DISPATCH_BOOL(hadamard, HAD,
        norm_gate_residual_kernel<CPT, true, true, HAD><<<(unsigned)rows, l.threads, 0, st>>>(
            (const uint16_t*)x, ldx, (const uint16_t*)r, ldr, (const uint16_t*)gate, ld_gate, rows_per_batch,
            w, (uint16_t*)y, ldy, w2, (const uint16_t*)scale, (const uint16_t*)shift, ld_mod, (int8_t*)q, ldq,
            (uint16_t*)sx, n, eps, eps2)));
  return zib_check_launch("norm_gate_residual_mod_quant");
}

extern "C" int zib_norm_gate_residual_mod_quant_w16(const void* x, int64_t ldx, const void* r, int64_t ldr,
                                                    const void* gate, int64_t ld_gate, int64_t rows_per_batch,
                                                    const void* w, void* y, int64_t ldy,
                                                    const void* w2, const void* scale, const void* shift,
                                                    int64_t ld_mod, void* q, int64_t ldq, void* sx,
                                                    int64_t rows, int64_t n, float eps, float eps2,
                                                    int hadamard, void* stream) {
  ZIB_HOST_CHECK(x && r && gate && w && y && w2 && scale && q && sx, ZIB_ERR_INVALID_ARG,
                 "norm_gate_residual_mod_quant_w16: null pointer");
  ZIB_HOST_CHECK(rows >= 0 && n == 3840 && rows_per_batch > 0, ZIB_ERR_INVALID_ARG,
                 "norm_gate_residual_mod_quant_w16: rows of 3840 features only (n=%lld)", (long long)n);
  ZIB_HOST_CHECK(ldx % 8 == 0 && ldr % 8 == 0 && ldy % 8 == 0 && ld_gate % 8 == 0 && ld_mod % 8 == 0 &&
                     ldq % 8 == 0 && aligned16(x) && aligned16(r) && aligned16(y) && aligned16(gate) &&
                     aligned16(w) && aligned16(w2) && aligned16(scale) && aligned16(q) && (!shift || aligned16(shift)),
                 ZIB_ERR_ALIGNMENT, "norm_gate_residual_mod_quant_w16: misaligned operand");
  if (rows == 0) return ZIB_OK;
  cudaStream_t st = (cudaStream_t)stream;
  auto k = hadamard ? wr::ngr_rg<5, true, true> : wr::ngr_rg<5, false, true>;
  k<<<wr::grid_rg(k, 96, 1, rows), 96, 0, st>>>(
      (const uint16_t*)x, ldx, (const uint16_t*)r, ldr, (const uint16_t*)gate, ld_gate, rows_per_batch, w,
      (uint16_t*)y, ldy, w2, (const uint16_t*)scale, (const uint16_t*)shift, ld_mod, (int8_t*)q, ldq,
      (uint16_t*)sx, n, eps, eps2, rows);
  return zib_check_launch("norm_gate_residual_mod_quant_w16");
}

extern "C" int zib_swiglu(const void* gate, int64_t ldg, const void* up, int64_t ldu, void* out,
                          int64_t ldo, int64_t rows, int64_t n, void* stream) {
  ZIB_HOST_CHECK(gate && up && out, ZIB_ERR_INVALID_ARG, "swiglu: null pointer");
  ZIB_HOST_CHECK(rows >= 0 && n > 0 && ldg >= n && ldu >= n && ldo >= n, ZIB_ERR_INVALID_ARG, "swiglu: bad shape");
  if (rows == 0) return ZIB_OK;
  RowLaunch l;
  ZIB_HOST_CHECK(row_launch((n + 7) / 8, &l), ZIB_ERR_TOO_LARGE,
                 "Cannot launch kernel since n = %lld exceeds the maximum fused size 65536.", (long long)n);
  const bool vec = n % 8 == 0 && ldg % 8 == 0 && ldu % 8 == 0 && ldo % 8 == 0 && aligned16(gate) &&
                   aligned16(up) && aligned16(out);
  cudaStream_t st = (cudaStream_t)stream;
  bool launched = false;
  if (vec)
    launched = wr::dispatch(n, [&](auto Rc, int cpl) {
      constexpr int R = decltype(Rc)::value;
      auto k = wr::swiglu_wr<R, false, false>;
      k<<<wr::grid_for(k, R, cpl, 0, rows), 32 * wr::warps_of(R), 0, st>>>(
          (const uint16_t*)gate, ldg, (const uint16_t*)up, ldu, (uint16_t*)out, ldo, nullptr, 0, nullptr, cpl, rows);
    });
  if (vec && !launched)
    ZIB_DISPATCH_W(pipe::pipe_warps(n), ZIB_PIPE_TRY((pipe::swiglu_pipe<W, false, false>), 1, rows, n,
        (const uint16_t*)gate, ldg, (const uint16_t*)up, ldu, (uint16_t*)out, ldo, nullptr, 0, nullptr, n));
  if (!launched)
    ZIB_DISPATCH_CPT(l.cpt, ZIB_DISPATCH_BOOL(vec, VEC,
        swiglu_kernel<CPT, VEC, false, false><<<(unsigned)rows, l.threads, 0, st>>>(
            (const uint16_t*)gate, ldg, (const uint16_t*)up, ldu, (uint16_t*)out, ldo, nullptr, 0, nullptr, n)));
  return zib_check_launch("swiglu");
}

extern "C" int zib_swiglu_quant(const void* gate, int64_t ldg, const void* up, int64_t ldu,
                                void* q, int64_t ldq, void* sx, int64_t rows, int64_t n,
                                int hadamard, void* stream) {
  ZIB_HOST_CHECK(gate && up && q && sx, ZIB_ERR_INVALID_ARG, "swiglu_quant: null pointer");
  ZIB_HOST_CHECK(rows >= 0 && n > 0 && n % 8 == 0 && (!hadamard || n % kGroup == 0), ZIB_ERR_INVALID_ARG,
                 "swiglu_quant: bad shape n=%lld", (long long)n);
  ZIB_HOST_CHECK(ldg % 8 == 0 && ldu % 8 == 0 && ldq % 8 == 0 && aligned16(gate) && aligned16(up) && aligned16(q),
                 ZIB_ERR_ALIGNMENT, "swiglu_quant: misaligned operand");
  if (rows == 0) return ZIB_OK;
  RowLaunch l;
  ZIB_HOST_CHECK(row_launch(n / 8, &l), ZIB_ERR_TOO_LARGE, "swiglu_quant: n too large");
  cudaStream_t st = (cudaStream_t)stream;
  bool launched = wr::dispatch(n, [&](auto Rc, int cpl) {
    constexpr int R = decltype(Rc)::value;
    auto k = hadamard ? wr::swiglu_wr<R, true, true> : wr::swiglu_wr<R, true, false>;
    wr::set_smem(k, wr::smem_for(R, cpl, 1));
    k<<<wr::grid_for(k, R, cpl, 1, rows), 32 * wr::warps_of(R), wr::smem_for(R, cpl, 1), st>>>(
        (const uint16_t*)gate, ldg, (const uint16_t*)up, ldu, nullptr, 0, (int8_t*)q, ldq, (uint16_t*)sx, cpl, rows);
  });
  if (!launched)
  ZIB_DISPATCH_W(pipe::pipe_warps(n), ZIB_DISPATCH_BOOL(hadamard, HAD,
      ZIB_PIPE_TRY((pipe::swiglu_pipe<W, true, HAD>), 1, rows, n,
          (const uint16_t*)gate, ldg, (const uint16_t*)up, ldu, nullptr, 0, (int8_t*)q, ldq, (uint16_t*)sx, n)));
  if (!launched)
    ZIB_DISPATCH_CPT(l.cpt, ZIB_DISPATCH_BOOL(hadamard, HAD,
        swiglu_kernel<CPT, true, true, HAD><<<(unsigned)rows, l.threads, 0, st>>>(
            (const uint16_t*)gate, ldg, (const uint16_t*)up, ldu, nullptr, 0, (int8_t*)q, ldq, (uint16_t*)sx, n)));
  return zib_check_launch("swiglu_quant");
}

extern "C" int zib_qknorm_rope(const void* x, int64_t x_sb, int64_t x_ss, int64_t x_sh,
                               void* out, int64_t o_sb, int64_t o_ss, int64_t o_sh,
                               const float* cosp, const float* sinp, int64_t cs_b,
                               const float* w, int64_t B, int64_t S, int64_t H, int64_t d,
                               float eps, void* stream) {
  ZIB_HOST_CHECK(x && out && cosp && sinp, ZIB_ERR_INVALID_ARG, "qknorm_rope: null pointer");
  ZIB_HOST_CHECK(d == 128, ZIB_ERR_INVALID_ARG, "qknorm_rope: head_dim must be 128, got %lld", (long long)d);
  ZIB_HOST_CHECK(B >= 0 && S >= 0 && H >= 0, ZIB_ERR_INVALID_ARG, "qknorm_rope: bad shape");
  ZIB_HOST_CHECK(aligned16(x) && aligned16(out) && aligned16(cosp) && aligned16(sinp) && (!w || aligned16(w)) &&
                     x_sb % 8 == 0 && x_ss % 8 == 0 && x_sh % 8 == 0 && o_sb % 8 == 0 && o_ss % 8 == 0 &&
                     o_sh % 8 == 0 && cs_b % 4 == 0,
                 ZIB_ERR_ALIGNMENT, "qknorm_rope: operands must be 16-byte aligned");
  const int64_t tokens = B * S;
  if (tokens == 0 || H == 0) return ZIB_OK;
  // one warp per token, 8 warps per CTA, as many CTAs as fit (a grid-stride loop takes the rest)
  const int64_t need = (tokens + 7) / 8;
  const int64_t cap = (int64_t)pipe::num_sms() * 8;
  const unsigned blocks = (unsigned)(need < cap ? need : cap);
  cudaStream_t st = (cudaStream_t)stream;
  if (w) {
    qknorm_rope_kernel<true><<<blocks, 256, 0, st>>>(
        (const uint16_t*)x, x_sb, x_ss, x_sh, (uint16_t*)out, o_sb, o_ss, o_sh, cosp, sinp, cs_b, w, S, H, tokens, eps);
  } else {
    qknorm_rope_kernel<false><<<blocks, 256, 0, st>>>(
        (const uint16_t*)x, x_sb, x_ss, x_sh, (uint16_t*)out, o_sb, o_ss, o_sh, cosp, sinp, cs_b, w, S, H, tokens, eps);
  }
  return zib_check_launch("qknorm_rope");
}

extern "C" int zib_adaln_modulation(const void* raw, int64_t ldr, void* scale_msa, void* gate_msa,
                                    void* scale_mlp, void* gate_mlp, int64_t rows, int64_t dim, void* stream) {
  ZIB_HOST_CHECK(raw && scale_msa && gate_msa && scale_mlp && gate_mlp, ZIB_ERR_INVALID_ARG,
                 "adaln_modulation: null pointer");
  ZIB_HOST_CHECK(rows >= 0 && dim > 0 && ldr >= 4 * dim, ZIB_ERR_INVALID_ARG, "adaln_modulation: bad shape");
  const int64_t total = rows * dim;
  if (total == 0) return ZIB_OK;
  adaln_modulation_kernel<<<(unsigned)((total + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      (const uint16_t*)raw, ldr, (uint16_t*)scale_msa, (uint16_t*)gate_msa, (uint16_t*)scale_mlp,
      (uint16_t*)gate_mlp, rows, dim);
  return zib_check_launch("adaln_modulation");
}

extern "C" int zib_adaln_gates(const void* raw, int64_t ldr, void* gates, int64_t rows, int64_t dim,
                               void* stream) {
  ZIB_HOST_CHECK(raw && gates, ZIB_ERR_INVALID_ARG, "adaln_gates: null pointer");
  ZIB_HOST_CHECK(rows >= 0 && dim > 0 && ldr >= 4 * dim, ZIB_ERR_INVALID_ARG, "adaln_gates: bad shape");
  const int64_t total = rows * 2 * dim;
  if (total == 0) return ZIB_OK;
  adaln_gates_kernel<<<(unsigned)((total + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      (const uint16_t*)raw, ldr, (uint16_t*)gates, rows, dim);
  return zib_check_launch("adaln_gates");
}

extern "C" int zib_weight_prep(const void* w, int64_t ldw, void* wq, int64_t ldq, void* sw,
                               void* sw_f32, float* w_rot, int64_t ld_rot, int64_t N, int64_t K,
                               int hadamard, void* stream) {
  ZIB_HOST_CHECK(w && wq && sw, ZIB_ERR_INVALID_ARG, "weight_prep: null pointer");
  ZIB_HOST_CHECK(N >= 0 && K > 0 && K % 8 == 0 && (!hadamard || K % kGroup == 0), ZIB_ERR_INVALID_ARG,
                 "weight_prep: bad shape N=%lld K=%lld", (long long)N, (long long)K);
  ZIB_HOST_CHECK(ldw % 8 == 0 && ldq % 8 == 0 && aligned16(w) && aligned16(wq) &&
                     (!w_rot || (aligned16(w_rot) && ld_rot % 4 == 0 && ld_rot >= K)),
                 ZIB_ERR_ALIGNMENT, "weight_prep: misaligned operand");
  if (N == 0) return ZIB_OK;
  RowLaunch l;
  ZIB_HOST_CHECK(row_launch(K / 8, &l), ZIB_ERR_TOO_LARGE, "weight_prep: K too large");
  cudaStream_t st = (cudaStream_t)stream;
  ZIB_DISPATCH_CPT(l.cpt, ZIB_DISPATCH_BOOL(hadamard, HAD,
      weight_prep_kernel<CPT, HAD><<<(unsigned)N, l.threads, 0, st>>>(
          (const uint16_t*)w, ldw, (int8_t*)wq, ldq, (uint16_t*)sw, (float*)sw_f32, w_rot, ld_rot, K)));
  return zib_check_launch("weight_prep");
}
