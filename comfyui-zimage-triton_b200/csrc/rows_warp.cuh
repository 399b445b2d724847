// Warp-per-row kernels: R warps per row (R = 1 for 3840 columns, 4 for
// 10240; the fused norm kernels take teams of 3 for 3840), one read of every
// input and one write of every output.
//
// Lane l of warp r in a row's team owns the 16-byte chunks (8 bf16)
//   c = 32 * cpl * r + l + 32 * k,   k = 0 .. cpl-1,
// so every load and store instruction of a warp moves 512 contiguous bytes
// and a 128-element Hadamard group (16 chunks) sits in lanes 0-15 or 16-31 of
// one k (px::fwht128: 3 butterfly stages in-thread, 4 over xor shuffles; the
// same adds in the same order as the other rotation kernels, two fp32 lanes
// per packed instruction).  A row is copied
// into this warp's slice of shared memory with cp.async (chunk k of lane l at
// [k][l], conflict-free; all of a row's copies in flight at once, no
// registers held), and the heavy stages (norm, rotation, quantisation) are
// rolled loops over it, which keeps the code small enough for the
// instruction cache.  Row reductions are warp shuffles (plus one named
// barrier across the R warps); there are no CTA-wide barriers.  Arithmetic and rounding points are those of the kernels
// these replace (rms_norm.py:47-57, fused_norm_residual.py:58-73,
// int8_linear.py:119-130); packed bf16x2 multiplies / adds are used only where
// both operands are bf16, where the single rounding of the exact result equals
// the reference's fp32 operation rounded to bf16.
#pragma once

#include <type_traits>

namespace wr {

constexpr int kWarps = 4;  // warps per CTA when R divides it; a CTA runs kWarps / R rows at a time

// warps per CTA for teams of R warps: kWarps when R divides it, else one team
__host__ __device__ constexpr int warps_of(int R) { return kWarps % R == 0 ? kWarps : R; }

// --- packed bf16x2 helpers --------------------------------------------------------

__device__ __forceinline__ float lo_f(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float hi_f(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ uint32_t cvt2(float lo, float hi) {  // round each to bf16 (RNE)
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t hadd2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
// RN_bf16(a * b + c) per lane, one rounding
__device__ __forceinline__ uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}
__device__ __forceinline__ void unpack8(const uint4& d, float v[8]) {
  v[0] = lo_f(d.x); v[1] = hi_f(d.x); v[2] = lo_f(d.y); v[3] = hi_f(d.y);
  v[4] = lo_f(d.z); v[5] = hi_f(d.z); v[6] = lo_f(d.w); v[7] = hi_f(d.w);
}
__device__ __forceinline__ uint4 ld_nc(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }

// row / rows_per_batch, in 32 bits whenever both fit (the common case)
__device__ __forceinline__ int64_t batch_of(int64_t row, int64_t rows_per_batch) {
  if ((uint64_t)row <= 0xFFFFFFFFull && (uint64_t)rows_per_batch <= 0xFFFFFFFFull)
    return (int64_t)((uint32_t)row / (uint32_t)rows_per_batch);
  return row / rows_per_batch;
}

// --- team of R warps working on one row ---------------------------------------------

template <int R>
struct Team {
  int lane, wig, grp;
  __device__ __forceinline__ Team() {
    lane = threadIdx.x & 31;
    const int w = threadIdx.x >> 5;
    wig = w % R;
    grp = w / R;
  }
  __device__ __forceinline__ void sync() const {
    // barrier 1 + team (a constant when the CTA is one team)
    if (R > 1) asm volatile("bar.sync %0, %1;" ::"r"(warps_of(R) == R ? 1 : 1 + grp), "r"(R * 32) : "memory");
  }
  // exact in practice: every partial is an exact fp64 sum of fp32 chunk sums
  __device__ __forceinline__ double sum(double v, double* red) const {
    v = warp_sum_f64(v);
    if (R == 1) return v;
    if (lane == 0) red[threadIdx.x >> 5] = v;
    sync();
    double r = 0.0;
#pragma unroll
    for (int k = 0; k < R; ++k) r += red[grp * R + k];
    sync();
    return r;
  }
  __device__ __forceinline__ uint32_t umax(uint32_t v, uint32_t* red) const {
    v = __reduce_max_sync(0xFFFFFFFFu, v);
    if (R == 1) return v;
    if (lane == 0) red[threadIdx.x >> 5] = v;
    sync();
    uint32_t r = 0;
#pragma unroll
    for (int k = 0; k < R; ++k) r = max(r, red[grp * R + k]);
    sync();
    return r;
  }
  __device__ __forceinline__ int64_t chunk(int cpl, int k) const { return (int64_t)(wig * cpl + k) * 32 + lane; }
  // element offset of this lane's first chunk in a row; chunk k is at + 256 * k
  __device__ __forceinline__ int64_t first(int cpl) const { return ((int64_t)wig * cpl * 32 + lane) * 8; }
};

// Rotation pass over this warp's chunks of a row (slots base[0 .. 32*cpl)):
// each step takes 64 chunks, four 128-groups of 16 chunks, and gives a group
// to 8 lanes with two chunks each (i and i + 8: fwht128_pair, three shuffle
// stages instead of four).  `src(c)` produces the bf16 chunk c to rotate;
// the rotated chunk goes back to slot c, into the |max|, and to `sink(c, v)`.
// Lanes of a group past the end work on chunks 0-15 and discard the results
// (every lane must take part in the shuffles).  The slots are read and written
// across lanes: the caller syncs the warp before and after.
template <class Src, class Sink>
__device__ __forceinline__ void rotate_pairs(uint4* base, int cpl, int lane, px::AbsMax& am, const Src& src,
                                             const Sink& sink) {
  const int n = 32 * cpl;
  const int off = 16 * (lane >> 3) + (lane & 7);
#pragma unroll 1
  for (int c0 = 0; c0 < n; c0 += 64) {
    const bool valid = c0 + off < n;  // whole 16-chunk groups: chunk i valid <=> chunk i + 8 valid
    const int ca = valid ? c0 + off : (lane & 7);
    px::f2 A[4], B[4];
    px::fwht128_pair(src(ca), src(ca + 8), A, B, lane);
    const uint4 ra = px::had_round(A), rb = px::had_round(B);
    if (valid) {
      base[ca] = ra;
      base[ca + 8] = rb;
      am.add(ra);
      am.add(rb);
      sink(ca, ra);
      sink(ca + 8, rb);
    }
  }
}

struct NoSink {
  __device__ __forceinline__ void operator()(int, const uint4&) const {}
};

// rotate (optional) chunk d in place and fold its |max| (bf16 bits)
template <bool HAD>
__device__ __forceinline__ void rot_amax(uint4& d, px::AbsMax& am, int lane) {
  if (HAD) {
    px::f2 P[4];
    px::fwht128(d, P, lane);
    d = px::had_round(P);
  }
  am.add(d);
}

// bf16(y * bf16(1 + s)) (+ h) with the chunk's scale s and shift h already loaded
__device__ __forceinline__ uint4 modulate(const uint4& y, const uint4& s, const uint4& h, bool has_shift) {
  constexpr uint32_t kOne2 = 0x3F803F80u;  // bf16 (1.0, 1.0)
  uint4 r = make_uint4(hmul2(y.x, hadd2(kOne2, s.x)), hmul2(y.y, hadd2(kOne2, s.y)),
                       hmul2(y.z, hadd2(kOne2, s.z)), hmul2(y.w, hadd2(kOne2, s.w)));
  if (has_shift) r = make_uint4(hadd2(r.x, h.x), hadd2(r.y, h.y), hadd2(r.z, h.z), hadd2(r.w, h.w));
  return r;
}

// --- kernels ---------------------------------------------------------------------------

// this warp's slice of the CTA's dynamic shared memory: `nbuf` row buffers of
// cpl * 32 chunks each; returns this lane's slot in buffer 0 (buffer j at + j*cpl*32)
__device__ __forceinline__ uint4* warp_slice(int cpl, int nbuf) {
  extern __shared__ __align__(16) uint4 wr_smem[];
  return wr_smem + (threadIdx.x >> 5) * nbuf * cpl * 32 + (threadIdx.x & 31);
}

// issue the copies of this lane's cpl chunks of a row into its slots
__device__ __forceinline__ void copy_row(const uint16_t* __restrict__ src, uint4* sl, int cpl) {
  const uint32_t dst = (uint32_t)__cvta_generic_to_shared(sl);
#pragma unroll 4
  for (int k = 0; k < cpl; ++k)
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst + 512u * k), "l"(src + 256 * k)
                 : "memory");
}

// pull this warp's part of a row into L2 ahead of its copies (one bulk
// prefetch by lane 0; rows are 16-byte aligned)
template <int R>
__device__ __forceinline__ void prefetch_row(const Team<R>& t, const uint16_t* row_base, int cpl) {
  if (t.lane == 0)
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(row_base + (int64_t)t.wig * cpl * 256),
                 "r"((uint32_t)cpl * 512u)
                 : "memory");
}

// wait for this lane's copies (each lane reads back only its own slots)
__device__ __forceinline__ void copies_done() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// this lane's part of the row's sum of squares: its chunks' canonical fp32 sums, added in fp64
__device__ __forceinline__ double row_sumsq(const uint4* sl, int cpl) {
  double ss = 0.0;
#pragma unroll 4
  for (int k = 0; k < cpl; ++k) ss += px::sumsq_chunk(sl[32 * k]);
  return ss;
}

// quantise the rotated row in the warp slice, store q and sx (int8_linear.py:129-130)
template <int R>
__device__ __forceinline__ void quant_row(const Team<R>& t, const uint4* sl, int cpl, uint32_t m2, uint32_t* redu,
                                          int64_t row, int8_t* __restrict__ q, int64_t ldq,
                                          uint16_t* __restrict__ sx) {
  uint32_t m = max(m2 & 0xFFFFu, m2 >> 16);
  m = t.umax(m, redu);
  const float s = act_scale(__uint_as_float(m << 16));
  const float rcp = __fdiv_rn(1.0f, s);
  int8_t* qr = q + row * ldq + t.first(cpl);
  if (m < 0x7F80u) {  // finite |max| (a row-uniform branch)
#pragma unroll 1
    for (int k = 0; k < cpl; ++k) *reinterpret_cast<uint2*>(qr + 256 * k) = px::quant_chunk_rne(sl[32 * k], rcp);
  } else {
#pragma unroll 1
    for (int k = 0; k < cpl; ++k) *reinterpret_cast<uint2*>(qr + 256 * k) = px::quant_chunk(sl[32 * k], rcp);
  }
  if (t.wig == 0 && t.lane == 0) sx[row] = float_to_bf16_bits(s);
}

template <int R, bool HAD>
__global__ void __launch_bounds__(32 * warps_of(R)) act_quant_wr(const uint16_t* __restrict__ x, int64_t ldx,
                                                            int8_t* __restrict__ q, int64_t ldq,
                                                            uint16_t* __restrict__ sx, uint16_t* __restrict__ xr,
                                                            int cpl, int64_t rows) {
  __shared__ uint32_t redu[warps_of(R)];
  const Team<R> t;
  const int64_t f0 = t.first(cpl);
  uint4* sl = warp_slice(cpl, 1);
  const int64_t step = (int64_t)gridDim.x * (warps_of(R) / R);
  for (int64_t row = (int64_t)blockIdx.x * (warps_of(R) / R) + t.grp; row < rows; row += step) {
    // this warp's next row into L2 (measured: helps the plain quantiser, slows the rotating kernels)
    if (!HAD && row + step < rows) prefetch_row(t, x + (row + step) * ldx, cpl);
    copy_row(x + row * ldx + f0, sl, cpl);
    copies_done();
    px::AbsMax m;
    if (HAD) {
      uint4* base = sl - t.lane;
      uint16_t* xrr = xr ? xr + row * ldq + (f0 - 8 * t.lane) : nullptr;  // optional rotated copy
      __syncwarp();  // chunks copied by other lanes
      rotate_pairs(base, cpl, t.lane, m, [&](int c) { return base[c]; },
                   [&](int c, const uint4& v) {
                     if (xrr) *reinterpret_cast<uint4*>(xrr + 8 * c) = v;
                   });
      __syncwarp();
    } else {
#pragma unroll 1
      for (int k = 0; k < cpl; ++k) {
        const uint4 d = sl[32 * k];
        m.add(d);
        if (xr) *reinterpret_cast<uint4*>(xr + row * ldq + f0 + 256 * k) = d;  // optional copy
      }
    }
    quant_row<R>(t, sl, cpl, m.packed(), redu, row, q, ldq, sx);
    __syncwarp();
  }
}

// MODE 0: rmsnorm -> bf16; 1: rmsnorm * (1+s) (+shift) -> bf16; 2: MODE 1 -> rotate / quant
template <int R, int MODE, bool HAD>
__global__ void __launch_bounds__(32 * warps_of(R)) rmsnorm_wr(
    const uint16_t* __restrict__ x, int64_t ldx, const float* __restrict__ w, const uint16_t* __restrict__ scale,
    const uint16_t* __restrict__ shift, int64_t ld_mod, int64_t rows_per_batch, uint16_t* __restrict__ y,
    int64_t ldy, int8_t* __restrict__ q, int64_t ldq, uint16_t* __restrict__ sx, int64_t n, float eps, int cpl,
    int64_t rows) {
  __shared__ double redd[warps_of(R)];
  __shared__ uint32_t redu[warps_of(R)];
  const Team<R> t;
  const int64_t f0 = t.first(cpl);
  const float* wl = w + f0;
  uint4* sl = warp_slice(cpl, 1);
  const int64_t step = (int64_t)gridDim.x * (warps_of(R) / R);
  for (int64_t row = (int64_t)blockIdx.x * (warps_of(R) / R) + t.grp; row < rows; row += step) {
    copy_row(x + row * ldx + f0, sl, cpl);
    copies_done();
    const float rstd = rstd_from_sum(t.sum(row_sumsq(sl, cpl), redd), (int)n, eps);
    const int64_t mo = batch_of(row, rows_per_batch) * ld_mod + f0;
    uint16_t* yr = MODE <= 1 ? y + row * ldy + f0 : nullptr;
    px::AbsMax m;
    if (MODE == 2 && HAD) {
      uint4* base = sl - t.lane;
      const int64_t c0 = f0 - 8 * t.lane, m0 = mo - 8 * t.lane;  // element offsets of the warp's chunk 0
      __syncwarp();  // chunks copied by other lanes
      rotate_pairs(base, cpl, t.lane, m,
                   [&](int c) {
                     return modulate(px::norm_w(base[c], rstd, w + c0 + 8 * c), ld_nc(scale + m0 + 8 * c),
                                     shift ? ld_nc(shift + m0 + 8 * c) : make_uint4(0, 0, 0, 0), shift != nullptr);
                   },
                   NoSink{});
      __syncwarp();
    } else
#pragma unroll 1
    for (int k = 0; k < cpl; ++k) {
      uint4 v = px::norm_w(sl[32 * k], rstd, wl + 256 * k);
      if (MODE >= 1)
        v = modulate(v, ld_nc(scale + mo + 256 * k), shift ? ld_nc(shift + mo + 256 * k) : make_uint4(0, 0, 0, 0),
                     shift != nullptr);
      if (MODE <= 1) {
        *reinterpret_cast<uint4*>(yr + 256 * k) = v;
      } else {
        rot_amax<HAD>(v, m, t.lane);
        sl[32 * k] = v;
      }
    }
    if (MODE == 2) quant_row<R>(t, sl, cpl, m.packed(), redu, row, q, ldq, sx);
    __syncwarp();  // the slot is rewritten by the next row's copies
  }
}

// row buffers per warp of ngr_wr: the residual row is staged for teams of three
__host__ __device__ constexpr int ngr_buffers(int R) { return R == 3 ? 2 : 1; }

// y = r + g * rmsnorm(x); FUSE: then rmsnorm(y; w2) * (1+s) (+shift) -> rotate / quant.
// Teams of three warps (R = 3, picked for 3840 features) copy the residual row
// into a second row buffer together with x, so that both rows are in flight at
// once; otherwise the residual is loaded chunk by chunk after the first norm's
// reduction.  Measured at [9216, 3840] on B200: one warp per row 94 us; teams
// of three 86 us (a row's latency split three ways, with a third of a row's
// buffer per warp); the staged residual 86 us fused, 47 -> 45 us unfused; with
// one warp per row the doubled buffer halves the resident warps and costs 22 us.
template <int R, bool FUSE, bool HAD>
__global__ void __launch_bounds__(32 * warps_of(R)) ngr_wr(
    const uint16_t* __restrict__ x, int64_t ldx, const uint16_t* __restrict__ r, int64_t ldr,
    const uint16_t* __restrict__ gate, int64_t ld_gate, int64_t rows_per_batch, const float* __restrict__ w,
    uint16_t* __restrict__ y, int64_t ldy, const float* __restrict__ w2, const uint16_t* __restrict__ scale,
    const uint16_t* __restrict__ shift, int64_t ld_mod, int8_t* __restrict__ q, int64_t ldq,
    uint16_t* __restrict__ sx, int64_t n, float eps, float eps2, int cpl, int64_t rows) {
  __shared__ double redd[warps_of(R)];
  __shared__ uint32_t redu[warps_of(R)];
  const Team<R> t;
  const int64_t f0 = t.first(cpl);
  const float* wl = w + f0;
  constexpr bool STAGE = R == 3;
  uint4* sl = warp_slice(cpl, ngr_buffers(R));  // x, then y
  uint4* se = sl + 32 * cpl;                    // STAGE: the residual row
  const int64_t step = (int64_t)gridDim.x * (warps_of(R) / R);
  for (int64_t row = (int64_t)blockIdx.x * (warps_of(R) / R) + t.grp; row < rows; row += step) {
    const uint16_t* rr = r + row * ldr + f0;
    copy_row(x + row * ldx + f0, sl, cpl);
    if (STAGE) {
      asm volatile("cp.async.commit_group;" ::: "memory");
      copy_row(rr, se, cpl);
      asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 1;" ::: "memory");  // x has landed
    } else {
      copies_done();
    }
    const float rstd = rstd_from_sum(t.sum(row_sumsq(sl, cpl), redd), (int)n, eps);
    const int64_t b = batch_of(row, rows_per_batch);
    const uint16_t* gl = gate + b * ld_gate + f0;
    uint16_t* yr = y + row * ldy + f0;
    double ss2 = 0.0;
    if (STAGE) asm volatile("cp.async.wait_group 0;" ::: "memory");  // the residual row has landed
#pragma unroll 4
    for (int k = 0; k < cpl; ++k) {
      const uint4 e = STAGE ? se[32 * k] : __ldcs(reinterpret_cast<const uint4*>(rr + 256 * k));
      const uint4 a = px::norm_w(sl[32 * k], rstd, wl + 256 * k);
      const uint4 g = ld_nc(gl + 256 * k);
      // RN_bf16(r + g * a), one rounding: the reference's compiler contracts the bf16
      // multiply-add of fused_norm_residual.py:72 into a fused multiply-add
      const uint4 v = make_uint4(hfma2(g.x, a.x, e.x), hfma2(g.y, a.y, e.y),
                                 hfma2(g.z, a.z, e.z), hfma2(g.w, a.w, e.w));
      *reinterpret_cast<uint4*>(yr + 256 * k) = v;
      if (FUSE) {
        sl[32 * k] = v;
        ss2 += px::sumsq_chunk(v);
      }
    }
    if (FUSE) {
      const float rstd2 = rstd_from_sum(t.sum(ss2, redd), (int)n, eps2);
      const int64_t mo = b * ld_mod + f0;
      const float* w2l = w2 + f0;
      px::AbsMax m;
      // one chunk per lane here: the paired rotation measured 2% slower in this kernel
#pragma unroll 1
      for (int k = 0; k < cpl; ++k) {
        uint4 v = modulate(px::norm_w(sl[32 * k], rstd2, w2l + 256 * k), ld_nc(scale + mo + 256 * k),
                           shift ? ld_nc(shift + mo + 256 * k) : make_uint4(0, 0, 0, 0), shift != nullptr);
        rot_amax<HAD>(v, m, t.lane);
        sl[32 * k] = v;
      }
      quant_row<R>(t, sl, cpl, m.packed(), redu, row, q, ldq, sx);
    }
    __syncwarp();
  }
}

// --- register-resident rows ------------------------------------------------------------
//
// The same kernels for the two row widths of the DiT step (3840 features: teams
// of three warps, five chunks per lane; 10240: teams of four, ten chunks), with
// the row held in registers: every input chunk of a row is loaded once, at the
// start of the row, with all of them in flight together; nothing is staged in
// shared memory (which only carries the team reductions), and the chunk loops
// are unrolled (CPL is a template argument).  The chunk ownership, the
// arithmetic and its order are those of the shared-memory kernels above, so
// the results are the same bits.  Measured on B200 (kernel medians, L2 flushed):
// the fused norm kernel at [9216, 3840] 85 -> 72 us (staged in shared memory it
// ran at 80% of the L1 data pipe: each staged row written once and read four
// times), the plain quantiser at [9216, 10240] 65 -> 51 us, the rotating one at
// [9216, 3840] 39 -> 37 us, norm + modulation + quantisation 57 -> 51 us.  The
// SwiGLU quantiser (two 10240-wide inputs) measured slower this way and keeps
// the shared-memory kernel.  A 128-group per quad of lanes (32 elements per
// lane, a quarter of the transform's shuffles) measured slower again: its
// 64-byte runs per lane take four times the L1 wavefronts per load.

// a 16-byte load of streamed data (read once): not kept in L1, where the norm
// weights and modulation vectors that every row reads stay
__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 v;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(p));
  return v;
}

// Team size and chunks per lane of the register-resident kernels for a row of n bf16
__host__ __device__ constexpr bool rg_shape(int64_t n, int* R, int* cpl) {
  if (n == 3840) { *R = 3; *cpl = 5; return true; }
  if (n == 10240) { *R = 4; *cpl = 10; return true; }
  return false;
}

// quant_row on the team's rotated chunks held in registers
template <int R, int CPL>
__device__ __forceinline__ void quant_regs(const Team<R>& t, const uint4 (&v)[CPL], uint32_t m2, uint32_t* redu,
                                           int64_t row, int8_t* __restrict__ q, int64_t ldq,
                                           uint16_t* __restrict__ sx) {
  uint32_t m = max(m2 & 0xFFFFu, m2 >> 16);
  m = t.umax(m, redu);
  const float s = act_scale(__uint_as_float(m << 16));
  const float rcp = __fdiv_rn(1.0f, s);
  int8_t* qr = q + row * ldq + t.first(CPL);
  if (m < 0x7F80u) {  // finite |max| (a row-uniform branch)
#pragma unroll
    for (int k = 0; k < CPL; ++k) *reinterpret_cast<uint2*>(qr + 256 * k) = px::quant_chunk_rne(v[k], rcp);
  } else {
#pragma unroll
    for (int k = 0; k < CPL; ++k) *reinterpret_cast<uint2*>(qr + 256 * k) = px::quant_chunk(v[k], rcp);
  }
  if (t.wig == 0 && t.lane == 0) sx[row] = float_to_bf16_bits(s);
}

// act_quant_wr with the row in registers
template <int R, int CPL, bool HAD>
__global__ void __launch_bounds__(32 * warps_of(R)) act_quant_rg(const uint16_t* __restrict__ x, int64_t ldx,
                                                            int8_t* __restrict__ q, int64_t ldq,
                                                            uint16_t* __restrict__ sx, uint16_t* __restrict__ xr,
                                                            int64_t rows) {
  __shared__ uint32_t redu[warps_of(R)];
  const Team<R> t;
  const int64_t f0 = t.first(CPL);
  const int64_t step = (int64_t)gridDim.x * (warps_of(R) / R);
  for (int64_t row = (int64_t)blockIdx.x * (warps_of(R) / R) + t.grp; row < rows; row += step) {
    const uint16_t* xp = x + row * ldx + f0;
    uint4 v[CPL];
#pragma unroll
    for (int k = 0; k < CPL; ++k) v[k] = ld_stream(xp + 256 * k);
    px::AbsMax m;
#pragma unroll
    for (int k = 0; k < CPL; ++k) {
      rot_amax<HAD>(v[k], m, t.lane);
      if (xr) *reinterpret_cast<uint4*>(xr + row * ldq + f0 + 256 * k) = v[k];  // optional copy
    }
    quant_regs<R, CPL>(t, v, m.packed(), redu, row, q, ldq, sx);
  }
}

// the chunk's norm with the weights at element offset e of w: fp32 (norm_w) or bf16 (W16: norm_w16)
template <bool W16>
__device__ __forceinline__ uint4 norm_any(const uint4& d, float rstd, const void* __restrict__ w, int64_t e) {
  if (W16) return px::norm_w16(d, rstd, ld_nc(reinterpret_cast<const uint16_t*>(w) + e));
  return px::norm_w(d, rstd, reinterpret_cast<const float*>(w) + e);
}

// ngr_wr<3, true, HAD> (norm + gate + residual, then norm * (1+s) (+shift) ->
// rotate / quantise) with the rows x and r in registers; W16: the norm weights w, w2 are
// bf16 (half the L1 traffic of fp32 weights, which take two half-sector loads per chunk)
template <int CPL, bool HAD, bool W16>
__global__ void __launch_bounds__(96) ngr_rg(
    const uint16_t* __restrict__ x, int64_t ldx, const uint16_t* __restrict__ r, int64_t ldr,
    const uint16_t* __restrict__ gate, int64_t ld_gate, int64_t rows_per_batch, const void* __restrict__ w,
    uint16_t* __restrict__ y, int64_t ldy, const void* __restrict__ w2, const uint16_t* __restrict__ scale,
    const uint16_t* __restrict__ shift, int64_t ld_mod, int8_t* __restrict__ q, int64_t ldq,
    uint16_t* __restrict__ sx, int64_t n, float eps, float eps2, int64_t rows) {
  constexpr int R = 3;
  static_assert(warps_of(R) == R, "one team per CTA");
  __shared__ double redd[R];
  __shared__ uint32_t redu[R];
  const Team<R> t;
  const int64_t f0 = t.first(CPL);
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    uint4 a[CPL], e[CPL];
#pragma unroll
    for (int k = 0; k < CPL; ++k) a[k] = ld_stream(x + row * ldx + f0 + 256 * k);
#pragma unroll
    for (int k = 0; k < CPL; ++k) e[k] = ld_stream(r + row * ldr + f0 + 256 * k);
    double ss = 0.0;
#pragma unroll
    for (int k = 0; k < CPL; ++k) ss += px::sumsq_chunk(a[k]);
    const float rstd = rstd_from_sum(t.sum(ss, redd), (int)n, eps);
    const int64_t b = batch_of(row, rows_per_batch);
    const uint16_t* gl = gate + b * ld_gate + f0;
    uint16_t* yr = y + row * ldy + f0;
    double ss2 = 0.0;
#pragma unroll
    for (int k = 0; k < CPL; ++k) {
      const uint4 nv = norm_any<W16>(a[k], rstd, w, f0 + 256 * k);
      const uint4 g = ld_nc(gl + 256 * k);
      // RN_bf16(r + g * a), one rounding, as in ngr_wr
      a[k] = make_uint4(hfma2(g.x, nv.x, e[k].x), hfma2(g.y, nv.y, e[k].y), hfma2(g.z, nv.z, e[k].z),
                        hfma2(g.w, nv.w, e[k].w));
      *reinterpret_cast<uint4*>(yr + 256 * k) = a[k];
      ss2 += px::sumsq_chunk(a[k]);
    }
    const float rstd2 = rstd_from_sum(t.sum(ss2, redd), (int)n, eps2);
    const int64_t mo = b * ld_mod + f0;
    px::AbsMax m;
#pragma unroll
    for (int k = 0; k < CPL; ++k) {
      a[k] = modulate(norm_any<W16>(a[k], rstd2, w2, f0 + 256 * k), ld_nc(scale + mo + 256 * k),
                      shift ? ld_nc(shift + mo + 256 * k) : make_uint4(0, 0, 0, 0), shift != nullptr);
      rot_amax<HAD>(a[k], m, t.lane);
    }
    quant_regs<R, CPL>(t, a, m.packed(), redu, row, q, ldq, sx);
  }
}

// rmsnorm_wr<R, 2, HAD> (norm * (1+s) (+shift) -> rotate / quantise) with the row in registers
template <int R, int CPL, bool HAD>
__global__ void __launch_bounds__(32 * warps_of(R)) rmsnorm_mod_quant_rg(
    const uint16_t* __restrict__ x, int64_t ldx, const float* __restrict__ w, const uint16_t* __restrict__ scale,
    const uint16_t* __restrict__ shift, int64_t ld_mod, int64_t rows_per_batch, int8_t* __restrict__ q, int64_t ldq,
    uint16_t* __restrict__ sx, int64_t n, float eps, int64_t rows) {
  __shared__ double redd[warps_of(R)];
  __shared__ uint32_t redu[warps_of(R)];
  const Team<R> t;
  const int64_t f0 = t.first(CPL);
  const int64_t step = (int64_t)gridDim.x * (warps_of(R) / R);
  for (int64_t row = (int64_t)blockIdx.x * (warps_of(R) / R) + t.grp; row < rows; row += step) {
    uint4 a[CPL];
#pragma unroll
    for (int k = 0; k < CPL; ++k) a[k] = ld_stream(x + row * ldx + f0 + 256 * k);
    double ss = 0.0;
#pragma unroll
    for (int k = 0; k < CPL; ++k) ss += px::sumsq_chunk(a[k]);
    const float rstd = rstd_from_sum(t.sum(ss, redd), (int)n, eps);
    const int64_t mo = batch_of(row, rows_per_batch) * ld_mod + f0;
    px::AbsMax m;
#pragma unroll
    for (int k = 0; k < CPL; ++k) {
      a[k] = modulate(px::norm_w(a[k], rstd, w + f0 + 256 * k), ld_nc(scale + mo + 256 * k),
                      shift ? ld_nc(shift + mo + 256 * k) : make_uint4(0, 0, 0, 0), shift != nullptr);
      rot_amax<HAD>(a[k], m, t.lane);
    }
    quant_regs<R, CPL>(t, a, m.packed(), redu, row, q, ldq, sx);
  }
}

// CTAs for a register-resident kernel (no dynamic shared memory): all that fit, at most one per team-row
template <class K>
static int grid_rg(K kernel, int threads, int rows_per_cta, int64_t rows) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, 0) != cudaSuccess || per_sm < 1) {
    cudaGetLastError();
    per_sm = 1;
  }
  const int64_t need = (rows + rows_per_cta - 1) / rows_per_cta;
  const int64_t g = (int64_t)per_sm * pipe::num_sms();
  return (int)(need < g ? need : g);
}

// out = bf16(bf16(silu(g)) * u) (swiglu.py:51-58); QUANT: then rotate (HAD) and
// quantise the row (int8_linear.py:119-130) instead of storing it.  silu and the
// product are the packed forms of the SwiGLU GEMM epilogue (same roundings as
// the scalar fp32 ones: the product of two bf16 values is exact in fp32).
template <int R, bool QUANT, bool HAD>
__global__ void __launch_bounds__(32 * warps_of(R)) swiglu_wr(
    const uint16_t* __restrict__ g, int64_t ldg, const uint16_t* __restrict__ u, int64_t ldu,
    uint16_t* __restrict__ out, int64_t ldo, int8_t* __restrict__ q, int64_t ldq, uint16_t* __restrict__ sx,
    int cpl, int64_t rows) {
  __shared__ uint32_t redu[warps_of(R)];
  const Team<R> t;
  const int64_t f0 = t.first(cpl);
  uint4* sl = QUANT ? warp_slice(cpl, 1) : nullptr;
  const int64_t step = (int64_t)gridDim.x * (warps_of(R) / R);
  for (int64_t row = (int64_t)blockIdx.x * (warps_of(R) / R) + t.grp; row < rows; row += step) {
    const uint16_t* gr = g + row * ldg + f0;
    const uint16_t* ur = u + row * ldu + f0;
    px::AbsMax m;
#pragma unroll 4
    for (int k = 0; k < cpl; ++k) {
      const uint4 gv = ld_nc(gr + 256 * k), uv = ld_nc(ur + 256 * k);
      const uint4 v =
          make_uint4(hmul2(px::silu_bf16x2(gv.x), uv.x), hmul2(px::silu_bf16x2(gv.y), uv.y),
                     hmul2(px::silu_bf16x2(gv.z), uv.z), hmul2(px::silu_bf16x2(gv.w), uv.w));
      if (!QUANT) {
        *reinterpret_cast<uint4*>(out + row * ldo + f0 + 256 * k) = v;
      } else {
        sl[32 * k] = v;
        if (!HAD) m.add(v);
      }
    }
    if (QUANT) {
      if (HAD) {
        uint4* base = sl - t.lane;
        __syncwarp();  // chunks written by other lanes
        rotate_pairs(base, cpl, t.lane, m, [&](int c) { return base[c]; }, NoSink{});
        __syncwarp();
      }
      quant_row<R>(t, sl, cpl, m.packed(), redu, row, q, ldq, sx);
      __syncwarp();
    }
  }
}

// --- host side ---------------------------------------------------------------------------

// Team size and chunks per lane for a row of n bf16: n % 256 == 0 and at most
// 16 chunks (8 KB of shared memory per row buffer) per warp; `three` asks for
// teams of three warps where they fit; false -> the caller uses another kernel.
static inline bool pick(int64_t n, bool three, int* R, int* cpl) {
  if (n <= 0 || n % 256) return false;
  const int64_t t = n / 256;
  if (three && t % 3 == 0 && t / 3 <= 16) {
    *R = 3;
    *cpl = (int)(t / 3);
    return true;
  }
  for (int r = 1; r <= 4; r *= 2) {
    if (t % r == 0 && t / r <= 16) {
      *R = r;
      *cpl = (int)(t / r);
      return true;
    }
  }
  return false;
}

// dynamic shared memory of a CTA: warps_of(R) slices of nbuf row buffers of cpl * 32 chunks
static inline size_t smem_for(int R, int cpl, int nbuf) { return (size_t)warps_of(R) * nbuf * cpl * 32 * 16; }

template <class K>
static int grid_for(K kernel, int R, int cpl, int nbuf, int64_t rows) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, 32 * warps_of(R), smem_for(R, cpl, nbuf)) !=
          cudaSuccess ||
      per_sm < 1) {
    cudaGetLastError();
    per_sm = 1;
  }
  const int64_t per_cta = warps_of(R) / R;
  const int64_t need = (rows + per_cta - 1) / per_cta;
  const int64_t g = (int64_t)per_sm * pipe::num_sms();
  return (int)(need < g ? need : g);
}

template <class K>
static void set_smem(K kernel, size_t bytes) {
  if (bytes > 48 * 1024) cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

// Calls f(integral_constant<R>, cpl) for the team size picked for n (THREE:
// teams of three warps where they fit); false when n has no warp-row shape.
template <bool THREE = false, class F>
static bool dispatch(int64_t n, F&& f) {
  int R, cpl;
  if (!pick(n, THREE, &R, &cpl)) return false;
  using std::integral_constant;
  if constexpr (THREE) {
    if (R == 3) {
      f(integral_constant<int, 3>{}, cpl);
      return true;
    }
  }
  if (R == 1) f(integral_constant<int, 1>{}, cpl);
  else if (R == 2) f(integral_constant<int, 2>{}, cpl);
  else f(integral_constant<int, 4>{}, cpl);
  return true;
}

}  // namespace wr
