// Bandwidth-bound row kernels of the Z-Image W8A8 path (sm_100a).
//
// One CTA processes one row.  A row is split into 8-element chunks; chunk c
// is owned by thread (c mod blockDim), so a 128-element Hadamard group is
// held by 16 consecutive lanes (8 values each) and rotated with 3 in-thread
// butterfly stages plus 4 xor-shuffle stages.  Every kernel keeps the
// reference's bf16 rounding points; see zib_common.cuh.
#include "zib_common.cuh"

#include <stdio.h>

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
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += (double)(v[i][j] * v[i][j]);  // exact products
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
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += (double)(v[i][j] * v[i][j]);
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
        float t = bf16_round(__fmul_rn(gv[j], xs));
        v[i][j] = bf16_round(__fadd_rn(rv[j], t));
        if (FUSE) ss2 += (double)(v[i][j] * v[i][j]);
      }
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
// 16 lanes per (token, head) row, 8 values (4 pairs) per lane.
// ---------------------------------------------------------------------------
template <bool NORM>
__global__ void __launch_bounds__(256) qknorm_rope_kernel(
    const uint16_t* __restrict__ x, int64_t x_sb, int64_t x_ss, int64_t x_sh,
    uint16_t* __restrict__ out, int64_t o_sb, int64_t o_ss, int64_t o_sh,
    const float* __restrict__ cosp, const float* __restrict__ sinp, int64_t cs_b,
    const float* __restrict__ w, int64_t S, int64_t H, int64_t total_rows, float eps) {
  const int lane = threadIdx.x & 31;
  const int sub = lane & 15;
  const int64_t rowg = (int64_t)blockIdx.x * (blockDim.x / 16) + (threadIdx.x >> 4);
  const bool valid = rowg < total_rows;
  const int64_t rr = valid ? rowg : 0;
  const int64_t h = rr % H;
  const int64_t t = rr / H;
  const int64_t s = t % S;
  const int64_t b = t / S;
  float v[8];
  load_bf16x8(x + b * x_sb + s * x_ss + h * x_sh + sub * 8, v);
  if (NORM) {
    double ss = 0.0;
#pragma unroll
    for (int j = 0; j < 8; ++j) ss += (double)(v[j] * v[j]);
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
    const float rstd = rstd_from_sum(ss, 128, eps);
    float4 wa = __ldg(reinterpret_cast<const float4*>(w + sub * 8));
    float4 wb = __ldg(reinterpret_cast<const float4*>(w + sub * 8 + 4));
    const float wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = bf16_round(__fmul_rn(bf16_round(__fmul_rn(v[j], rstd)), wv[j]));
  }
  const float4 c4 = __ldg(reinterpret_cast<const float4*>(cosp + b * cs_b + s * 64 + sub * 4));
  const float4 s4 = __ldg(reinterpret_cast<const float4*>(sinp + b * cs_b + s * 64 + sub * 4));
  const float cv[4] = {c4.x, c4.y, c4.z, c4.w};
  const float sv[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float a = v[2 * k], bb = v[2 * k + 1];
    v[2 * k] = bf16_round(__fsub_rn(__fmul_rn(a, cv[k]), __fmul_rn(bb, sv[k])));
    v[2 * k + 1] = bf16_round(__fadd_rn(__fmul_rn(bb, cv[k]), __fmul_rn(a, sv[k])));
  }
  if (valid) store_bf16x8(out + b * o_sb + s * o_ss + h * o_sh + sub * 8, v);
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

}  // namespace zib

using namespace zib;

#define ZIB_DISPATCH_CPT(cpt, ...)              \
  switch (cpt) {                                \
    case 1: { constexpr int CPT = 1; __VA_ARGS__; } break; \
    case 2: { constexpr int CPT = 2; __VA_ARGS__; } break; \
    case 4: { constexpr int CPT = 4; __VA_ARGS__; } break; \
    default: { constexpr int CPT = 8; __VA_ARGS__; } break; \
  }

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
  ZIB_DISPATCH_CPT(l.cpt, ZIB_DISPATCH_BOOL(hadamard, HAD,
      norm_gate_residual_kernel<CPT, true, true, HAD><<<(unsigned)rows, l.threads, 0, st>>>(
          (const uint16_t*)x, ldx, (const uint16_t*)r, ldr, (const uint16_t*)gate, ld_gate, rows_per_batch,
          w, (uint16_t*)y, ldy, w2, (const uint16_t*)scale, (const uint16_t*)shift, ld_mod, (int8_t*)q, ldq,
          (uint16_t*)sx, n, eps, eps2)));
  return zib_check_launch("norm_gate_residual_mod_quant");
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
  const int64_t rows = B * S * H;
  if (rows == 0) return ZIB_OK;
  const int rows_per_block = 16;  // 256 threads
  const int64_t blocks = (rows + rows_per_block - 1) / rows_per_block;
  ZIB_HOST_CHECK(blocks < (1ll << 31), ZIB_ERR_TOO_LARGE, "qknorm_rope: too many rows");
  cudaStream_t st = (cudaStream_t)stream;
  if (w) {
    qknorm_rope_kernel<true><<<(unsigned)blocks, 256, 0, st>>>(
        (const uint16_t*)x, x_sb, x_ss, x_sh, (uint16_t*)out, o_sb, o_ss, o_sh, cosp, sinp, cs_b, w, S, H, rows, eps);
  } else {
    qknorm_rope_kernel<false><<<(unsigned)blocks, 256, 0, st>>>(
        (const uint16_t*)x, x_sb, x_ss, x_sh, (uint16_t*)out, o_sb, o_ss, o_sh, cosp, sinp, cs_b, w, S, H, rows, eps);
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
