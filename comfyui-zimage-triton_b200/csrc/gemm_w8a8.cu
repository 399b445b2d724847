// K1: W8A8 GEMM on 5th-generation tensor cores (tcgen05, kind::i8) for sm_100a.
//
// Replaces torch._int_mm plus the eager dequant epilogue of the reference's
// W8A8+Hadamard linear (src/zimage_triton/quantization/int8_linear.py:133-137):
//   acc[m,n] = sum_k q[m,k] * wq[n,k]                         (int32, exact)
//   y[m,n]   = bf16( bf16(acc) * bf16(sx[m] * sw[n]) ) (+ bias[n])
// and, as fused epilogues, the op that consumes the GEMM output in the block:
//   SWIGLU  x_rot = rot128( bf16( bf16(silu(g)) * u ) )   g = w1 output, u = w3 output
//           (swiglu.py:51-58, then int8_linear.py:119-126 for the w2 input)
//   QKROPE  per-head RMSNorm * w then interleaved RoPE on the Q and K heads of
//           the QKV output (fused_qknorm_rope.py:85-151), V unchanged.
//
// Design (persistent, warp-specialised, one CTA per SM):
//   warp 0      TMA producer (128-byte swizzled K-major tiles).
//   warp 1      owns TMEM (512 columns = two 128x256 int32 accumulators) and
//               issues tcgen05.mma from one thread.
//   warps 2..    epilogue (8 warps, 16 for SWIGLU): the NQ warps w, w+4, ...
//               read the same 32 accumulator rows (TMEM lane quarter w%4) and
//               split the 256 columns in NQ parts; accumulator buffer b is
//               drained while the MMA fills the other.
//   1-CTA tiles are 128x256 (48 KB stages).  For M > 128 a cluster of two
//   CTAs (cta_group::2) computes 256x256 tiles: each CTA stages its 128 A rows
//   and 128 of the B rows (32 KB stages), both CTAs' TMA loads complete on
//   the leader's barrier, the leader issues M=256 MMAs reading both CTAs'
//   shared memory, and its commits are multicast to both CTAs.  No TMA load
//   uses cluster multicast.
//   The fused epilogues run in two phases.  Phase 1, one thread per
//   accumulator row: TMEM -> dequant -> SwiGLU (or the row's sum of squares)
//   -> bf16 into a swizzled shared-memory tile, after which the accumulator
//   buffer is released to the MMA.  Phase 2, 16 lanes per row with 8 values
//   each (the row kernels' layout): the 128-point Hadamard transform on
//   shuffles (SWIGLU) or norm * w + RoPE with coalesced cos/sin (QKROPE), and
//   coalesced 256-byte row stores.
//   SWIGLU tiles stage 64 rows of each weight per 128 tile columns,
//   [w1 f0..f0+63 | w3 f0..f0+63 | w1 f0+64..f0+127 | w3 f0+64..f0+127], so
//   each column quarter pairs 32 gate columns with the up columns 64 further on.
// Every mbarrier wait is bounded (globaltimer); on expiry the CTA records
// ZIB_ERR_TIMEOUT in a device error word, drains its in-flight TMA loads and
// MMAs, frees TMEM and exits.
#include "zib_async.cuh"
#include "rot_pack.cuh"

#include <cuda.h>
#include <mutex>

ZIB_DEFINE_ERROR_READER(zib_err_read_clear_gemm)

namespace zib {
namespace gemm {

enum Epi : int { EPI_BF16 = 0, EPI_I32 = 1, EPI_SWIGLU = 2, EPI_QKROPE = 3 };

constexpr int BK = 128;  // bytes == int8 elements == one 128-byte swizzle row
constexpr int BN = 256;  // accumulator columns per tile
constexpr int UMMA_K = 32;
constexpr int HALF_BYTES = 128 * BK;  // one 128-row operand box
constexpr int TMEM_COLS = 512;
constexpr int SW_BOX_ROWS = 64;                // SWIGLU B box: 64 weight rows of w1 or of w3
constexpr int SW_BOX_BYTES = SW_BOX_ROWS * BK;
constexpr int S_STAGE_BYTES = 3 * HALF_BYTES;  // 1-CTA: A 128x128 + B 256x128
constexpr int P_STAGE_BYTES = 2 * HALF_BYTES;  // 2-CTA pair: A 128x128 + B 128x128 per CTA
constexpr int MAX_SMEM = 232448;

// Per-epilogue pipeline depth and shared-memory layout (from the 1024-aligned
// base): [stages][256 B barriers][XBUF bytes of epilogue staging].
template <int EPI>
struct Cfg {
  // warp 0 TMA, warp 1 MMA/TMEM, then EPI_WARPS epilogue warps (NQ per TMEM lane quarter)
  static constexpr int EPI_WARPS = EPI == EPI_SWIGLU ? 16 : 8;
  static constexpr int NQ = EPI_WARPS / 4;
  static constexpr int THREADS = (2 + EPI_WARPS) * 32;
  // SWIGLU: 128 rows x 128 features bf16.
  // QKROPE: 128 rows x 256 columns bf16.
  static constexpr int XBUF = EPI == EPI_SWIGLU ? 128 * 256 : (EPI == EPI_QKROPE ? 128 * 512 : 0);
  static constexpr int S_STAGES = EPI == EPI_QKROPE ? 3 : 4;
  static constexpr int P_STAGES = EPI == EPI_QKROPE ? 5 : (EPI == EPI_SWIGLU ? 6 : 7);
  static constexpr int S_SMEM = S_STAGES * S_STAGE_BYTES + 1024 + 256 + XBUF;
  static constexpr int P_SMEM = P_STAGES * P_STAGE_BYTES + 1024 + 256 + XBUF;
  static_assert(S_SMEM <= MAX_SMEM && P_SMEM <= MAX_SMEM, "shared memory per CTA");
};

// instruction descriptors: D=s32, A=B=s8, both K-major, N=256, M=128 / 256
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

struct Params {
  int M, N, K;  // N: output columns (SWIGLU: features)
  int num_mb, num_nb, num_kb, num_tiles;
  int n_fast;  // tile order: 0 = M-blocks fastest (B read once), 1 = N-blocks fastest (A read once)
  int group;   // blocks of the fast index per group (the tiles sweep one group at a time)
  const uint16_t* sx;
  const uint16_t* sw;   // per weight row (SWIGLU: w1 scales)
  const uint16_t* sw2;  // SWIGLU: w3 scales
  int w13;              // SWIGLU: B is one [2F, K] tensor, the F rows of w1 then the F rows of w3
  const uint16_t* bias;
  uint16_t* y;
  int64_t ldy;
  int st32;  // y rows 32-byte aligned (y and ldy): the plain epilogue stores whole 32-byte sectors
  int32_t* acc;
  int64_t ldacc;
  // QKROPE
  const float* qn_w;
  const float* kn_w;
  float q_eps, k_eps;
  const float* cosp;
  const float* sinp;
  int64_t cs_b;
  int seq, heads;
  // split-K tail (plain and int32 epilogues of the pair kernel): work units
  // [0, tail_start) are whole tiles; the remaining tiles run as `splits` units
  // each over a slice of K, whose int32 partial tiles meet in `ws`
  int num_units, tail_start, splits;
  // half tiles (pair kernel, plain and int32 epilogues, whole-K units only): the
  // tail tiles [tail_start, num_tiles) run as two units of 128 output columns each
  int halves;
  int32_t* ws;        // [tail tile][cta rank][split][128 x 256] int32 partials
  int* counters;      // [tail tile][cta rank] arrivals, back to 0 after the last one
};

// --- PTX wrappers ------------------------------------------------------------

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t mbar_cluster, int x,
                                                 int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
      "%4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(mbar_cluster), "r"(x), "r"(y)
      : "memory");
}

// 3-D box (x = k, y = row, z = which of the two stacked [F, K] halves)
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d_pair(void* dst, const CUtensorMap* map, uint32_t mbar_cluster, int x,
                                                 int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
      "%4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(mbar_cluster), "r"(x), "r"(y), "r"(z)
      : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// K-major operand tile written by TMA with 128-byte swizzle: rows of 128 bytes,
// 8-row core groups 1024 bytes apart (SBO), descriptor version 1.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}

__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void umma_i8_pair(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// arrive (when this thread's prior MMAs retire) on `bar` in every CTA of `mask`
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar, uint16_t mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(mask)
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// whole warp, converged: load 32 accumulator columns of this thread's row
__device__ __forceinline__ void tmem_row32(uint32_t taddr, uint32_t (&r)[32]) {
  __syncwarp();
  tmem_ld32(taddr, r);
  tmem_wait_ld();
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t mapa_rank(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// named barrier over the epilogue warps of one TMEM lane quarter (nthreads = 32 * NQ)
__device__ __forceinline__ void group_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// same barrier, returning the AND of `ok` over its threads
__device__ __forceinline__ int group_bar_and(int id, int nthreads, int ok) {
  int out;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 q, %1, 0;\n\t"
      "bar.red.and.pred p, %2, %3, q;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(out)
      : "r"(ok), "r"(id), "r"(nthreads)
      : "memory");
  return out;
}

// --- epilogues -----------------------------------------------------------------

// bf16 round-to-nearest-even on the ALU pipe (finite inputs); keeps the
// conversion pipe free for the int32 -> fp32 conversions.
__device__ __forceinline__ float bf16_rne_alu(float v) {
  uint32_t b = __float_as_uint(v);
  b += 0x7FFFu + ((b >> 16) & 1u);
  return __uint_as_float(b & 0xFFFF0000u);
}

// y = bf16( bf16(acc) * bf16(sx * sw) )   (int8_linear.py:134)
__device__ __forceinline__ float dequant(uint32_t acc, float sxf, float swf) {
  const float s = bf16_rne_alu(__fmul_rn(sxf, swf));
  const float a = bf16_rne_alu(__int2float_rn((int)acc));
  return bf16_rne_alu(__fmul_rn(a, s));
}

// Packed bf16x2 forms (low half = even column).  The product of two bf16
// values is exact in fp32, so mul.rn.bf16x2 (one rounding of the exact
// product) equals the reference's bf16 multiply (fp32 product, rounded).
__device__ __forceinline__ uint32_t cvt_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint32_t mul_bf16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ float lo_f32(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float hi_f32(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// dequant of columns (2i, 2i+1): sx2 = {sx, sx}, sw2 = {sw[2i], sw[2i+1]}
__device__ __forceinline__ uint32_t dequant2(uint32_t acc0, uint32_t acc1, uint32_t sx2, uint32_t sw2) {
  const uint32_t s2 = mul_bf16x2(sx2, sw2);
  const uint32_t a2 = cvt_bf16x2(__int2float_rn((int)acc0), __int2float_rn((int)acc1));
  return mul_bf16x2(a2, s2);
}

__device__ __forceinline__ uint4 ldg_u4(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }

__device__ __forceinline__ void store_row_bf16(uint16_t* dst, const float* v, int n) {
#pragma unroll
  for (int j = 0; j < n; j += 8) store_bf16x8(dst + j, v + j);
}

// Staging-tile offsets: 16-byte chunk c of tile row r, XOR-swizzled so that
// 8 consecutive rows writing the same chunk, and 8 consecutive chunks of one
// row, fall on distinct bank groups.
__device__ __forceinline__ uint32_t xoff_256(int r, int c) { return (uint32_t)(r * 256 + ((c ^ (r & 15)) << 4)); }
__device__ __forceinline__ uint32_t xoff_512(int r, int c) { return (uint32_t)(r * 512 + ((c ^ (r & 7)) << 4)); }

struct EpiCtx {
  uint32_t t_row;  // TMEM address: this warp's lane quarter in the current accumulator buffer
  int row_base;    // global row of tile row 0 in this CTA
  int quarter;     // TMEM lane quarter (warp % 4)
  int cq;          // column part: 256/NQ accumulator columns (warps 2..5 -> 0, 6..9 -> 1, ...)
  int lane;
  int bar_id;      // named barrier of this lane quarter's four warps
  uint8_t* xbuf;   // epilogue staging tile
};

// releases the accumulator buffer: 1-CTA (local barrier) or pair (leader's barrier)
struct ReleaseLocal {
  uint64_t* bar;
  __device__ __forceinline__ void operator()(int lane) const {
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(bar);
  }
};
struct ReleaseLeader {
  uint32_t bar_cluster;
  __device__ __forceinline__ void operator()(int lane) const {
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive_cluster(bar_cluster);
  }
};

// one 32-column chunk of plain dequant (+bias) or raw int32 output for one row
template <int EPI>
__device__ __forceinline__ void epi_chunk(const Params& p, int row, int n0, const uint32_t (&r)[32],
                                          uint32_t sx2, float sxf) {
  const bool full = n0 + 32 <= p.N;
  if (EPI == EPI_I32) {
    int32_t* dst = p.acc + (int64_t)row * p.ldacc + n0;
    if (full && (p.ldacc % 4) == 0) {
#pragma unroll
      for (int j = 0; j < 32; j += 4)
        *reinterpret_cast<int4*>(dst + j) = make_int4((int)r[j], (int)r[j + 1], (int)r[j + 2], (int)r[j + 3]);
    } else {
      for (int j = 0; j < 32 && n0 + j < p.N; ++j) dst[j] = (int)r[j];
    }
  } else if (full && !p.bias && p.st32) {
    // one 32-byte store per 16 columns: whole L2 sectors instead of two half-sector writes
    uint16_t* dst = p.y + (int64_t)row * p.ldy + n0;
#pragma unroll
    for (int j = 0; j < 32; j += 16) {
      const uint4 wa = ldg_u4(p.sw + n0 + j), wb = ldg_u4(p.sw + n0 + j + 8);
      const uint32_t o0 = dequant2(r[j], r[j + 1], sx2, wa.x), o1 = dequant2(r[j + 2], r[j + 3], sx2, wa.y);
      const uint32_t o2 = dequant2(r[j + 4], r[j + 5], sx2, wa.z), o3 = dequant2(r[j + 6], r[j + 7], sx2, wa.w);
      const uint32_t o4 = dequant2(r[j + 8], r[j + 9], sx2, wb.x), o5 = dequant2(r[j + 10], r[j + 11], sx2, wb.y);
      const uint32_t o6 = dequant2(r[j + 12], r[j + 13], sx2, wb.z), o7 = dequant2(r[j + 14], r[j + 15], sx2, wb.w);
      asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(dst + j), "r"(o0), "r"(o1),
                   "r"(o2), "r"(o3), "r"(o4), "r"(o5), "r"(o6), "r"(o7)
                   : "memory");
    }
  } else if (full && !p.bias) {
    uint16_t* dst = p.y + (int64_t)row * p.ldy + n0;
#pragma unroll
    for (int j = 0; j < 32; j += 8) {
      const uint4 w = ldg_u4(p.sw + n0 + j);
      uint4 o;
      o.x = dequant2(r[j], r[j + 1], sx2, w.x);
      o.y = dequant2(r[j + 2], r[j + 3], sx2, w.y);
      o.z = dequant2(r[j + 4], r[j + 5], sx2, w.z);
      o.w = dequant2(r[j + 6], r[j + 7], sx2, w.w);
      *reinterpret_cast<uint4*>(dst + j) = o;
    }
  } else {
    float out[32];
#pragma unroll
    for (int j = 0; j < 32; j += 8) {
      float swv[8], bv[8];
      if (full) {
        load_bf16x8_nc(p.sw + n0 + j, swv);
        if (p.bias) load_bf16x8_nc(p.bias + n0 + j, bv);
      } else {
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          const int n = n0 + j + t;
          swv[t] = n < p.N ? bf16_bits_to_float(p.sw[n]) : 0.0f;
          bv[t] = (p.bias && n < p.N) ? bf16_bits_to_float(p.bias[n]) : 0.0f;
        }
      }
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        float v = dequant(r[j + t], sxf, swv[t]);
        if (p.bias) v = bf16_rne_alu(__fadd_rn(v, bv[t]));
        out[j + t] = v;
      }
    }
    uint16_t* dst = p.y + (int64_t)row * p.ldy + n0;
    if (full) {
      store_row_bf16(dst, out, 32);
    } else {
      for (int j = 0; j < 32 && n0 + j < p.N; ++j) dst[j] = (uint16_t)(__float_as_uint(out[j]) >> 16);
    }
  }
}

// plain dequant (+bias) or raw int32: this thread's row, accumulator columns [32 * nch * cq, +32 * nch)
// of a unit whose column 0 is output column n_base
template <int EPI, class Rel>
__device__ __forceinline__ void epi_plain(const Params& p, const EpiCtx& c, int n_base, int nch, const Rel& rel) {
  const int row = c.row_base + c.quarter * 32 + c.lane;
  const bool row_ok = row < p.M;
  uint16_t sxb = 0;
  if (EPI == EPI_BF16 && row_ok) sxb = p.sx[row];
  const uint32_t sx2 = (uint32_t)sxb | ((uint32_t)sxb << 16);
  const float sxf = __uint_as_float((uint32_t)sxb << 16);
#pragma unroll 1
  for (int ch = c.cq * nch; ch < c.cq * nch + nch; ++ch) {
    uint32_t r[32];
    tmem_row32(c.t_row + (uint32_t)(ch * 32), r);
    const int n0 = n_base + ch * 32;
    if (!row_ok || n0 >= p.N) continue;
    epi_chunk<EPI>(p, row, n0, r, sx2, sxf);
  }
  rel(c.lane);
}

constexpr int kSplitBar = 6;  // named barrier over all epilogue warps of a CTA (ids 1-4: lane quarters)

// Split-K tail unit of the pair kernel (plain / int32 epilogues).  Every split
// stores its int32 partial for this CTA's 128 rows, releases the accumulator,
// and counts itself in; the split that arrives last for the tile (whichever
// it is) sums the partials of all splits and runs the ordinary epilogue on
// the sums.  Integer sums are exact in any order, so the output is the one
// the whole-K tile produces.  Partials are laid out [chunk][4-column group]
// [row] of int4 so that a warp's stores and loads are 512 contiguous bytes.
template <int EPI, class Rel>
__device__ __forceinline__ void epi_split(const Params& p, const EpiCtx& c, int nb, int tail_idx, int split,
                                          int rank, const Rel& rel) {
  __shared__ int s_last;
  constexpr int CH = 8 / Cfg<EPI>::NQ;
  const int rt = c.quarter * 32 + c.lane;
  int4* slots = reinterpret_cast<int4*>(p.ws + (int64_t)(tail_idx * 2 + rank) * p.splits * (128 * 256));
  constexpr int kSlotInt4 = 128 * 256 / 4;
#pragma unroll 1
  for (int ch = c.cq * CH; ch < c.cq * CH + CH; ++ch) {
    uint32_t r[32];
    tmem_row32(c.t_row + (uint32_t)(ch * 32), r);
    int4* dst = slots + (int64_t)split * kSlotInt4 + (ch * 8) * 128 + rt;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      __stcg(dst + j * 128, make_int4((int)r[4 * j], (int)r[4 * j + 1], (int)r[4 * j + 2], (int)r[4 * j + 3]));
  }
  rel(c.lane);
  __threadfence();
  group_bar_sync(kSplitBar, Cfg<EPI>::EPI_WARPS * 32);
  if (c.cq == 0 && c.quarter == 0 && c.lane == 0) {
    int* ctr = p.counters + tail_idx * 2 + rank;
    const int last = atomicAdd(ctr, 1) == p.splits - 1;
    if (last) *ctr = 0;  // every split of this tile has arrived: ready for the next launch
    s_last = last;
  }
  group_bar_sync(kSplitBar, Cfg<EPI>::EPI_WARPS * 32);
  if (!s_last) return;
  __threadfence();
  const int row = c.row_base + rt;
  const bool row_ok = row < p.M;
  uint16_t sxb = 0;
  if (EPI == EPI_BF16 && row_ok) sxb = p.sx[row];
  const uint32_t sx2 = (uint32_t)sxb | ((uint32_t)sxb << 16);
  const float sxf = __uint_as_float((uint32_t)sxb << 16);
#pragma unroll 1
  for (int ch = c.cq * CH; ch < c.cq * CH + CH; ++ch) {
    const int n0 = nb * BN + ch * 32;
    if (!row_ok || n0 >= p.N) continue;
    uint32_t r[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) r[j] = 0u;
#pragma unroll 1
    for (int sp = 0; sp < p.splits; ++sp) {
      const int4* src = slots + (int64_t)sp * kSlotInt4 + (ch * 8) * 128 + rt;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int4 v = __ldcg(src + j * 128);
        r[4 * j] += (uint32_t)v.x;
        r[4 * j + 1] += (uint32_t)v.y;
        r[4 * j + 2] += (uint32_t)v.z;
        r[4 * j + 3] += (uint32_t)v.w;
      }
    }
    epi_chunk<EPI>(p, row, n0, r, sx2, sxf);
  }
}

// SWIGLU.  Phase 1 (thread = row): the tile's 256 accumulator columns are two
// parts of [64 gate | 64 up] columns; column quarter cq holds gate (cols
// 128*(cq/2) + 32*(cq%2) + [0, 32)) and up (those + 64) of features 128*nb + 32*cq + [0, 32);
// the bf16 SwiGLU values go to the staging tile [128 rows][128 features].
// Phase 2 (8 lanes per row, two chunks each): Walsh-Hadamard over the 128
// features of a row (index bits 0..2 and 6 in-thread, 3..5 by xor shuffles,
// in the act_quant kernels' order), times bf16(1/sqrt(128)) correctly
// rounded, stored to x_rot.
template <class Rel>
__device__ __forceinline__ void epi_swiglu(const Params& p, const EpiCtx& c, int nb, const Rel& rel) {
  static_assert(Cfg<EPI_SWIGLU>::NQ == 4, "SWIGLU column quarters");
  const int rt = c.quarter * 32 + c.lane;
  const int row = c.row_base + rt;
  const uint32_t sxb = row < p.M ? (uint32_t)p.sx[row] : 0u;
  const uint32_t sx2 = sxb | (sxb << 16);
  const int fb = nb * 128 + c.cq * 32;
  const uint32_t tc = c.t_row + (uint32_t)((c.cq >> 1) * 128 + (c.cq & 1) * 32);
#pragma unroll 1
  for (int g = 0; g < 2; ++g) {
    uint32_t rg[16], ru[16];
    __syncwarp();
    tmem_ld16(tc + (uint32_t)(g * 16), rg);
    tmem_ld16(tc + (uint32_t)(SW_BOX_ROWS + g * 16), ru);
    tmem_wait_ld();
    const uint4 s1a = ldg_u4(p.sw + fb + g * 16), s1b = ldg_u4(p.sw + fb + g * 16 + 8);
    const uint4 s3a = ldg_u4(p.sw2 + fb + g * 16), s3b = ldg_u4(p.sw2 + fb + g * 16 + 8);
    const uint32_t s1[8] = {s1a.x, s1a.y, s1a.z, s1a.w, s1b.x, s1b.y, s1b.z, s1b.w};
    const uint32_t s3[8] = {s3a.x, s3a.y, s3a.z, s3a.w, s3b.x, s3b.y, s3b.z, s3b.w};
    uint32_t v[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const uint32_t g2 = dequant2(rg[2 * t], rg[2 * t + 1], sx2, s1[t]);
      const uint32_t u2 = dequant2(ru[2 * t], ru[2 * t + 1], sx2, s3[t]);
      // silu in fp32, rounded to bf16; times up, rounded to bf16 (swiglu.py:51-58)
      v[t] = mul_bf16x2(px::silu_bf16x2(g2), u2);
    }
    const int ch = c.cq * 4 + g * 2;
    *reinterpret_cast<uint4*>(c.xbuf + xoff_256(rt, ch)) = make_uint4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<uint4*>(c.xbuf + xoff_256(rt, ch + 1)) = make_uint4(v[4], v[5], v[6], v[7]);
  }
  rel(c.lane);  // accumulator read: the MMA may refill this buffer
  group_bar_sync(c.bar_id, 128);
  const int sub = c.lane & 7;  // 8 lanes per row, chunks sub and sub + 8 (fwht128_pair)
#pragma unroll 1
  for (int it = 0; it < 2; ++it) {
    const int r2 = c.quarter * 32 + c.cq * 8 + it * 4 + (c.lane >> 3);
    px::f2 A[4], B[4];
    px::fwht128_pair(*reinterpret_cast<const uint4*>(c.xbuf + xoff_256(r2, sub)),
                     *reinterpret_cast<const uint4*>(c.xbuf + xoff_256(r2, sub + 8)), A, B, c.lane);
    const uint4 oa = px::had_round(A), ob = px::had_round(B);
    const int grow = c.row_base + r2;
    if (grow < p.M) {
      uint16_t* dst = p.y + (int64_t)grow * p.ldy + nb * 128 + sub * 8;
      *reinterpret_cast<uint4*>(dst) = oa;
      *reinterpret_cast<uint4*>(dst + 64) = ob;
    }
  }
}

// QKROPE: the tile holds heads hb = 2*nb and 2*nb+1 of the [Q | K | V]
// projection (the head count is even, so both have the same kind); column
// part cq is tile columns [CW*cq, CW*cq + CW), CW = 256/NQ.
// Phase 1 (thread = row, one warp per head): dequantised columns -> staging
// tile, the row's exact sum of squares and its rstd.  Phase 2 (16 lanes per
// row, 8 values each, the row's rstd by shuffle from its phase-1 lane):
// bf16(bf16(x * rstd) * w), interleaved-pair RoPE, coalesced store.
template <class Rel>
__device__ __forceinline__ void epi_qkrope(const Params& p, const EpiCtx& c, int nb, const Rel& rel) {
  constexpr int NQ = Cfg<EPI_QKROPE>::NQ;
  constexpr int CW = 256 / NQ;        // columns per warp
  constexpr int WPH = NQ / 2;         // warps per head
  constexpr int RPW = 32 / WPH;       // phase-2 rows per warp
  static_assert(WPH == 1, "one epilogue warp per head: phase 1 completes each row's sum of squares");
  const int rt = c.quarter * 32 + c.lane;
  const int row = c.row_base + rt;
  const bool row_ok = row < p.M;
  const uint32_t sxb = row_ok ? (uint32_t)p.sx[row] : 0u;
  const uint32_t sx2 = sxb | (sxb << 16);
  const int n0 = nb * 256 + c.cq * CW;  // first output column of this part
  const int kind = (nb * 2) / p.heads;  // 0 Q, 1 K, 2 V
  const uint32_t tc = c.t_row + (uint32_t)(c.cq * CW);
  if (kind == 2) {
#pragma unroll 1
    for (int cc = 0; cc < CW / 32; ++cc) {
      uint32_t r[32];
      tmem_row32(tc + (uint32_t)(cc * 32), r);
      uint16_t* dst = p.y + (int64_t)row * p.ldy + n0 + cc * 32;
#pragma unroll
      for (int j = 0; j < 32; j += 8) {
        const uint4 w = ldg_u4(p.sw + n0 + cc * 32 + j);
        uint4 o;
        o.x = dequant2(r[j], r[j + 1], sx2, w.x);
        o.y = dequant2(r[j + 2], r[j + 3], sx2, w.y);
        o.z = dequant2(r[j + 4], r[j + 5], sx2, w.z);
        o.w = dequant2(r[j + 6], r[j + 7], sx2, w.w);
        if (row_ok) *reinterpret_cast<uint4*>(dst + j) = o;
      }
    }
    rel(c.lane);
    return;
  }
  double ss = 0.0;
#pragma unroll 1
  for (int cc = 0; cc < CW / 32; ++cc) {
    uint32_t r[32];
    tmem_row32(tc + (uint32_t)(cc * 32), r);
#pragma unroll
    for (int j = 0; j < 32; j += 8) {
      const uint4 w = ldg_u4(p.sw + n0 + cc * 32 + j);
      const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
      uint32_t o[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) o[t] = dequant2(r[j + 2 * t], r[j + 2 * t + 1], sx2, wv[t]);
      const uint4 ch = make_uint4(o[0], o[1], o[2], o[3]);
      ss += px::sumsq_chunk(ch);  // canonical chunk sums, added exactly
      *reinterpret_cast<uint4*>(c.xbuf + xoff_512(rt, (c.cq * CW + cc * 32 + j) / 8)) = ch;
    }
  }
  rel(c.lane);
  // one warp per head: this thread's row of the head is complete, so its rstd is
  // formed here once and handed to phase 2's lanes by shuffle
  const float eps = kind == 0 ? p.q_eps : p.k_eps;
  const float rs_own = rstd_from_sum(ss, 128, eps);
  // this row's offset in the cos/sin tables (batch bi, position si; 32-bit, checked on the host)
  const int gr_own = row_ok ? row : 0;
  const int tab_own = (gr_own / p.seq) * (int)p.cs_b + (gr_own % p.seq) * 64;
  __syncwarp();  // the staging rows this warp wrote are read back by other lanes of it
  const int sub = c.lane & 15;
  const int hh = c.cq / WPH;  // head within the tile
  const float* w = kind == 0 ? p.qn_w : p.kn_w;
  const float4 wa = __ldg(reinterpret_cast<const float4*>(w + sub * 8));
  const float4 wb = __ldg(reinterpret_cast<const float4*>(w + sub * 8 + 4));
  const px::f2 W[4] = {px::mk(wa.x, wa.y), px::mk(wa.z, wa.w), px::mk(wb.x, wb.y), px::mk(wb.z, wb.w)};
#pragma unroll 4
  for (int it = 0; it < RPW / 2; ++it) {
    const int r2 = c.quarter * 32 + (c.cq % WPH) * RPW + it * 2 + (c.lane >> 4);
    const int grow = c.row_base + r2;
    const int owner = it * 2 + (c.lane >> 4);  // row r2's phase-1 lane
    const int tab = __shfl_sync(0xFFFFFFFFu, tab_own, owner) + sub * 4;
    const float4 c4 = __ldg(reinterpret_cast<const float4*>(p.cosp + tab));
    const float4 s4 = __ldg(reinterpret_cast<const float4*>(p.sinp + tab));
    const uint4 xv = *reinterpret_cast<const uint4*>(c.xbuf + xoff_512(r2, hh * 16 + sub));
    const float rs = __shfl_sync(0xFFFFFFFFu, rs_own, owner);
    const px::f2 RS = px::mk(rs, rs);
    const float cv[4] = {c4.x, c4.y, c4.z, c4.w};
    const float sv[4] = {s4.x, s4.y, s4.z, s4.w};
    const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      // bf16(bf16(x * rstd) * w), then the pair rotation fma(a, c, -(b s)),
      // fma(b, c, a s) as the reference's compiler contracts it (fused_qknorm_rope.py:140-141);
      // scalar intrinsics, so that no other contraction can change a rounding
      const uint32_t n2 = px::to_bf16x2(px::mul(px::from_bf16x2(xw[k]), RS));
      const uint32_t m2 = px::to_bf16x2(px::mul(px::from_bf16x2(n2), W[k]));
      const float a = lo_f32(m2), b = hi_f32(m2);
      o[k] = cvt_bf16x2(__fmaf_rn(a, cv[k], -__fmul_rn(b, sv[k])), __fmaf_rn(b, cv[k], __fmul_rn(a, sv[k])));
    }
    if (grow < p.M)
      *reinterpret_cast<uint4*>(p.y + (int64_t)grow * p.ldy + (nb * 2 + hh) * 128 + sub * 8) =
          make_uint4(o[0], o[1], o[2], o[3]);
  }
}

template <int EPI, class Rel>
__device__ __forceinline__ void epilogue_tile(const Params& p, const EpiCtx& c, int nb, const Rel& rel) {
  if (EPI == EPI_SWIGLU) epi_swiglu(p, c, nb, rel);
  else if (EPI == EPI_QKROPE) epi_qkrope(p, c, nb, rel);
  else epi_plain<EPI>(p, c, nb * BN, 8 / Cfg<EPI>::NQ, rel);
}

// Stage the B rows of tile nb for this CTA (`part` 0/1 = which 128 tile
// columns; the 1-CTA kernel stages both).  Standard tiles: 128 consecutive
// weight rows.  SWIGLU tiles: 64 rows of w1, then the same 64 rows of w3 (two
// boxes from two tensors; one 3-D box when w1 and w3 are the halves of one tensor).
template <int EPI>
__device__ __forceinline__ void load_b_part(uint8_t* dst, const CUtensorMap* b0, const CUtensorMap* b1, int nb,
                                            int part, int kx, uint64_t* bar, uint32_t pair_bar, bool pair,
                                            bool w13) {
  if (EPI == EPI_SWIGLU) {
    const int f = nb * 128 + part * SW_BOX_ROWS;
    if (w13) {
      if (pair) tma_load_3d_pair(dst, b0, pair_bar, kx, f, 0);
      else tma_load_3d(dst, b0, bar, kx, f, 0);
    } else if (pair) {
      tma_load_2d_pair(dst, b0, pair_bar, kx, f);
      tma_load_2d_pair(dst + SW_BOX_BYTES, b1, pair_bar, kx, f);
    } else {
      tma_load_2d(dst, b0, bar, kx, f);
      tma_load_2d(dst + SW_BOX_BYTES, b1, bar, kx, f);
    }
  } else {
    if (pair) tma_load_2d_pair(dst, b0, pair_bar, kx, nb * 256 + part * 128);
    else tma_load_2d(dst, b0, bar, kx, nb * 256 + part * 128);
  }
}

// Tile t -> (M-block, N-block).  Consecutive tiles run concurrently on the
// persistent CTAs, so the fastest-varying block index decides which operand
// stays resident in L2 while the other one streams.  The fast index runs in
// groups of p.group blocks: the tiles sweep every block of the slow index for
// one group before the next group, so the resident part of that operand is
// one group's rows, not all of them (M = 18432: A is 70.8 MB, more than stays
// in L2 next to the streamed outputs).
__device__ __forceinline__ void tile_coords(const Params& p, int tile, int& mb, int& nb) {
  const int nfast = p.n_fast ? p.num_nb : p.num_mb, nslow = p.n_fast ? p.num_mb : p.num_nb;
  const int per_group = p.group * nslow;
  const int g = tile / per_group, r = tile - g * per_group;
  const int gsize = min(p.group, nfast - g * p.group);  // the last group may be smaller
  const int f = g * p.group + r % gsize, sl = r / gsize;
  if (p.n_fast) {
    nb = f;
    mb = sl;
  } else {
    mb = f;
    nb = sl;
  }
}

// Skinny GEMM for M <= 8 rows (the stacked adaLN linear: 2 rows x 460800
// columns x K = 256): a 128-row tensor-core tile would be 94% padding and the
// launch is a stream over the weights, so each half-warp takes one weight row
// (column of the output) at a time, forms the MR int32 dot products with dp4a
// (exact, like the int32 accumulators of the tcgen05 path) and runs the same
// dequant (+bias) arithmetic as that path's epilogue.  The A rows sit in
// shared memory; each lane keeps four weight loads in flight.
constexpr int kSkinnyMaxM = 8;
constexpr int kSkinnyMaxK = 4096;

template <int EPI, int MR>
__global__ void __launch_bounds__(256) gemm_w8a8_skinny_kernel(const int8_t* __restrict__ q, int64_t ldq,
                                                               const int8_t* __restrict__ w, int64_t ldw,
                                                               const Params p) {
  extern __shared__ uint4 a_s[];  // [MR][K / 16]
  const int kc = p.K / 16;
  for (int i = threadIdx.x; i < MR * kc; i += blockDim.x) {
    const int m = i / kc, c = i % kc;
    a_s[i] = m < p.M ? __ldg(reinterpret_cast<const uint4*>(q + (int64_t)m * ldq) + c) : make_uint4(0, 0, 0, 0);
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, half = lane >> 4, sub = lane & 15;
  const int64_t warp = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  float sxf[MR];
#pragma unroll
  for (int m = 0; m < MR; ++m) sxf[m] = (EPI == EPI_BF16 && m < p.M) ? bf16_bits_to_float(p.sx[m]) : 0.0f;
  // a warp covers 8 columns per step: column 8 * step + 2 j + half, j = 0..3 (warp-uniform loop)
  for (int64_t base = warp * 8; base < p.N; base += nwarps * 8) {
    int32_t acc[4][MR];
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int m = 0; m < MR; ++m) acc[j][m] = 0;
    for (int c = sub; c < kc; c += 16) {
      uint4 wv[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t n = base + 2 * j + half;
        wv[j] = n < p.N ? __ldg(reinterpret_cast<const uint4*>(w + n * ldw) + c) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int m = 0; m < MR; ++m) {
        const uint4 a = a_s[m * kc + c];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          int t = acc[j][m];
          t = __dp4a((int)wv[j].x, (int)a.x, t);
          t = __dp4a((int)wv[j].y, (int)a.y, t);
          t = __dp4a((int)wv[j].z, (int)a.z, t);
          t = __dp4a((int)wv[j].w, (int)a.w, t);
          acc[j][m] = t;
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int m = 0; m < MR; ++m) {
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) acc[j][m] += __shfl_xor_sync(0xFFFFFFFFu, acc[j][m], o);
      }
      const int64_t n = base + 2 * j + half;
      if (sub != 0 || n >= p.N) continue;
      if (EPI == EPI_I32) {
#pragma unroll
        for (int m = 0; m < MR; ++m)
          if (m < p.M) p.acc[(int64_t)m * p.ldacc + n] = acc[j][m];
      } else {
        const float swf = bf16_bits_to_float(p.sw[n]);
        const float bf = p.bias ? bf16_bits_to_float(p.bias[n]) : 0.0f;
#pragma unroll
        for (int m = 0; m < MR; ++m) {
          if (m >= p.M) continue;
          float v = dequant((uint32_t)acc[j][m], sxf[m], swf);
          if (p.bias) v = bf16_rne_alu(__fadd_rn(v, bf));
          p.y[(int64_t)m * p.ldy + n] = (uint16_t)(__float_as_uint(v) >> 16);
        }
      }
    }
  }
}

// Work unit u -> tile, K-block range, split index (-1: the whole K range) and
// half (-1: all 256 columns; 0 / 1: columns [0, 128) / [128, 256) of the tile).
struct Unit {
  int tile, kb0, kb1, split, half;
};
__device__ __forceinline__ Unit unit_of(const Params& p, int u) {
  if (u < p.tail_start) return Unit{u, 0, p.num_kb, -1, -1};
  const int v = u - p.tail_start;
  if (p.halves) return Unit{p.tail_start + (v >> 1), 0, p.num_kb, -1, v & 1};
  const int sp = v % p.splits;
  return Unit{p.tail_start + v / p.splits, sp * p.num_kb / p.splits, (sp + 1) * p.num_kb / p.splits, sp, -1};
}

// --- kernels -------------------------------------------------------------------

template <int EPI>
__global__ void __launch_bounds__(Cfg<EPI>::THREADS, 1)
    gemm_w8a8_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                     const __grid_constant__ CUtensorMap tmap_b2, const Params p) {
  constexpr int STAGES = Cfg<EPI>::S_STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * S_STAGE_BYTES);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + STAGES;
  uint64_t* tfull_bar = bars + 2 * STAGES;
  uint64_t* tempty_bar = bars + 2 * STAGES + 2;
  uint64_t* mma_done_bar = bars + 2 * STAGES + 4;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  uint8_t* xbuf = smem + STAGES * S_STAGE_BYTES + 256;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], Cfg<EPI>::EPI_WARPS);
    }
    mbar_init(mma_done_bar, 1);
    *abort_flag = 0;
    mbar_fence_init();
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
    if (EPI == EPI_SWIGLU) tma_prefetch_desc(&tmap_b2);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {  // ---- TMA producer
      int stage = 0;
      uint32_t phase = 0, pend_mask = 0, pend_parity = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        int mb, nb;
        tile_coords(p, tile, mb, nb);
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait_bounded(&empty_bar[stage], phase ^ 1u, abort_flag)) { ok = false; break; }
          uint8_t* st = smem + stage * S_STAGE_BYTES;
          mbar_arrive_expect_tx(&full_bar[stage], S_STAGE_BYTES);
          tma_load_2d(st, &tmap_a, &full_bar[stage], kb * BK, mb * 128);
          load_b_part<EPI>(st + HALF_BYTES, &tmap_b, &tmap_b2, nb, 0, kb * BK, &full_bar[stage], 0, false, p.w13);
          load_b_part<EPI>(st + 2 * HALF_BYTES, &tmap_b, &tmap_b2, nb, 1, kb * BK, &full_bar[stage], 0, false, p.w13);
          pend_mask |= 1u << stage;
          pend_parity = (pend_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      if (!ok)
        for (int s = 0; s < STAGES; ++s)
          if (pend_mask & (1u << s)) mbar_drain_wait(&full_bar[s], (pend_parity >> s) & 1u);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {  // ---- MMA issuer
      int stage = 0, accb = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      const uint32_t base = smem_u32(smem);
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        if (!mbar_wait_bounded(&tempty_bar[accb], acc_phase ^ 1u, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(accb * BN);
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait_bounded(&full_bar[stage], phase, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint64_t adesc = sdesc_sw128(base + stage * S_STAGE_BYTES);
          const uint64_t bdesc = sdesc_sw128(base + stage * S_STAGE_BYTES + HALF_BYTES);
#pragma unroll
          for (int k = 0; k < BK / UMMA_K; ++k)
            umma_i8(d_tmem, adesc + (uint64_t)((k * UMMA_K) >> 4), bdesc + (uint64_t)((k * UMMA_K) >> 4),
                    idesc_i8(128, 256), (kb | k) != 0 ? 1u : 0u);
          umma_commit(&empty_bar[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        umma_commit(&tfull_bar[accb]);
        accb ^= 1;
        if (accb == 0) acc_phase ^= 1u;
      }
      umma_commit(mma_done_bar);
      mbar_drain_wait(mma_done_bar, 0);
    }
    __syncwarp();
  } else {
    // ---- epilogue: warps w, w+4, ... share TMEM lane quarter w%4 and split the columns
    const int cq = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int bar_id = 1 + ((warp - 2) & 3);
    int accb = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
      int ok = 1;
      if (lane == 0) ok = mbar_wait_bounded(&tfull_bar[accb], acc_phase, abort_flag) ? 1 : 0;
      ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
      if (EPI == EPI_SWIGLU || EPI == EPI_QKROPE) ok = group_bar_and(bar_id, Cfg<EPI>::NQ * 32, ok);
      if (!ok) break;
      tc_fence_after();
      int mb, nb;
        tile_coords(p, tile, mb, nb);
      const EpiCtx c{tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(accb * BN), mb * 128, quarter,
                     cq, lane, bar_id, xbuf};
      epilogue_tile<EPI>(p, c, nb, ReleaseLocal{&tempty_bar[accb]});
      accb ^= 1;
      if (accb == 0) acc_phase ^= 1u;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                 : "memory");
}

template <int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Cfg<EPI>::THREADS, 1)
    gemm_w8a8_pair_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                          const __grid_constant__ CUtensorMap tmap_b2, const Params p) {
  constexpr int STAGES = Cfg<EPI>::P_STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * P_STAGE_BYTES);
  uint64_t* full_bar = bars;                     // leader's is used
  uint64_t* empty_bar = bars + STAGES;           // both
  uint64_t* tfull_bar = bars + 2 * STAGES;       // both
  uint64_t* tempty_bar = bars + 2 * STAGES + 2;  // leader's is used
  uint64_t* mma_done_bar = bars + 2 * STAGES + 4;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  uint8_t* xbuf = smem + STAGES * P_STAGE_BYTES + 256;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int cluster_id = blockIdx.x >> 1;
  const int nclusters = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 2 * Cfg<EPI>::EPI_WARPS);  // epilogue warps of both CTAs
    }
    mbar_init(mma_done_bar, 1);
    *abort_flag = 0;
    mbar_fence_init();
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
    if (EPI == EPI_SWIGLU) tma_prefetch_desc(&tmap_b2);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers are initialised before any cross-CTA signal
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  bool aborted = false;

  if (warp == 0) {
    if (lane == 0) {  // ---- TMA producer (both CTAs)
      int stage = 0;
      uint32_t phase = 0, pend_mask = 0, pend_parity = 0;
      bool ok = true;
      for (int u = cluster_id; u < p.num_units && ok; u += nclusters) {
        const Unit w = unit_of(p, u);
        int mb, nb;
        tile_coords(p, w.tile, mb, nb);
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!mbar_wait_bounded(&empty_bar[stage], phase ^ 1u, abort_flag)) { ok = false; break; }
          const uint32_t fb = smem_u32(&full_bar[stage]);
          // a half unit stages 64 weight rows per CTA (the tensor map tmap_b2 has 64-row boxes)
          if (leader) mbar_arrive_expect_tx(&full_bar[stage], w.half < 0 ? 2 * P_STAGE_BYTES : 3 * HALF_BYTES);
          const uint32_t fb_leader = leader ? fb : mapa_rank(fb, 0);
          uint8_t* st = smem + stage * P_STAGE_BYTES;
          tma_load_2d_pair(st, &tmap_a, fb_leader, kb * BK, mb * 256 + (int)rank * 128);
          if ((EPI == EPI_BF16 || EPI == EPI_I32) && w.half >= 0)
            tma_load_2d_pair(st + HALF_BYTES, &tmap_b2, fb_leader, kb * BK, nb * 256 + w.half * 128 + (int)rank * 64);
          else
            load_b_part<EPI>(st + HALF_BYTES, &tmap_b, &tmap_b2, nb, (int)rank, kb * BK, nullptr, fb_leader, true,
                             p.w13);
          pend_mask |= 1u << stage;
          pend_parity = (pend_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      if (!ok) {
        aborted = true;
        if (leader)
          for (int s = 0; s < STAGES; ++s)
            if (pend_mask & (1u << s)) mbar_drain_wait(&full_bar[s], (pend_parity >> s) & 1u);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0 && leader) {  // ---- MMA issuer (leader CTA only)
      int stage = 0, accb = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      const uint32_t base = smem_u32(smem);
      for (int u = cluster_id; u < p.num_units && ok; u += nclusters) {
        const Unit w = unit_of(p, u);
        if (!mbar_wait_bounded(&tempty_bar[accb], acc_phase ^ 1u, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(accb * BN);
        const uint32_t idesc = w.half < 0 ? idesc_i8(256, 256) : idesc_i8(256, 128);
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!mbar_wait_bounded(&full_bar[stage], phase, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint64_t adesc = sdesc_sw128(base + stage * P_STAGE_BYTES);
          const uint64_t bdesc = sdesc_sw128(base + stage * P_STAGE_BYTES + HALF_BYTES);
#pragma unroll
          for (int k = 0; k < BK / UMMA_K; ++k)
            umma_i8_pair(d_tmem, adesc + (uint64_t)((k * UMMA_K) >> 4), bdesc + (uint64_t)((k * UMMA_K) >> 4),
                         idesc, (kb != w.kb0 || k != 0) ? 1u : 0u);
          umma_commit_pair(&empty_bar[stage], (uint16_t)3);  // frees the stage in both CTAs
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        umma_commit_pair(&tfull_bar[accb], (uint16_t)3);
        accb ^= 1;
        if (accb == 0) acc_phase ^= 1u;
      }
      if (!ok) aborted = true;
      umma_commit_pair(mma_done_bar, (uint16_t)1);
      mbar_drain_wait(mma_done_bar, 0);
    }
    __syncwarp();
  } else {
    // ---- epilogue (both CTAs): warps w, w+4, ... share lane quarter w%4, split the columns
    const int cq = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int bar_id = 1 + ((warp - 2) & 3);
    int accb = 0;
    uint32_t acc_phase = 0;
    for (int u = cluster_id; u < p.num_units; u += nclusters) {
      const Unit w = unit_of(p, u);
      int ok = 1;
      if (lane == 0) ok = mbar_wait_bounded(&tfull_bar[accb], acc_phase, abort_flag) ? 1 : 0;
      ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
      // with split units in the launch, every epilogue warp of the CTA agrees on every unit, so
      // that no warp can be left alone at the split epilogue's barrier after another one stopped
      if (EPI == EPI_SWIGLU || EPI == EPI_QKROPE) ok = group_bar_and(bar_id, Cfg<EPI>::NQ * 32, ok);
      else if (p.splits > 1) ok = group_bar_and(kSplitBar, Cfg<EPI>::EPI_WARPS * 32, ok);
      if (!ok) { aborted = true; break; }
      tc_fence_after();
      int mb, nb;
      tile_coords(p, w.tile, mb, nb);
      const EpiCtx c{tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(accb * BN),
                     mb * 256 + (int)rank * 128, quarter, cq, lane, bar_id, xbuf};
      const ReleaseLeader rel{mapa_rank(smem_u32(&tempty_bar[accb]), 0)};
      if constexpr (EPI == EPI_BF16 || EPI == EPI_I32) {
        if (w.split >= 0) epi_split<EPI>(p, c, nb, w.tile - p.tail_start, w.split, (int)rank, rel);
        else if (w.half >= 0) epi_plain<EPI>(p, c, nb * BN + w.half * 128, 4 / Cfg<EPI>::NQ, rel);
        else epilogue_tile<EPI>(p, c, nb, rel);
      } else {
        epilogue_tile<EPI>(p, c, nb, rel);
      }
      accb ^= 1;
      if (accb == 0) acc_phase ^= 1u;
    }
  }

  // An aborted CTA gives copies still in flight (the peer's loads complete on
  // the leader's barrier) a bounded grace period before the CTAs leave.
  if (__syncthreads_or(aborted ? 1 : 0)) {
    const unsigned long long t0 = globaltimer();
    while (globaltimer() - t0 < 2000000ull) {
    }
  }
  tc_fence_before();
  cluster_sync_all();  // both CTAs are done with TMEM and with each other's barriers
  tc_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                 : "memory");
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// int8 [2, rows, inner]: two [rows, inner] halves stacked (row stride ld_bytes, the second
// half rows * ld_bytes after the first), boxes of 128 bytes x box_rows x both halves, 128B swizzle
static int make_map_halves(CUtensorMap* map, const void* base, int64_t inner, int64_t rows, int64_t ld_bytes,
                           uint32_t box_rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) {
    zib_set_error("gemm_w8a8: cuTensorMapEncodeTiled unavailable");
    return ZIB_ERR_UNSUPPORTED;
  }
  cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)rows, 2};
  cuuint64_t strides[2] = {(cuuint64_t)ld_bytes, (cuuint64_t)(ld_bytes * rows)};
  cuuint32_t box[3] = {(cuuint32_t)BK, box_rows, 2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    zib_set_error("gemm_w8a8: cuTensorMapEncodeTiled (3-D) failed (%d)", (int)r);
    return ZIB_ERR_INVALID_ARG;
  }
  return ZIB_OK;
}

// int8 [outer, inner] row-major with row stride ld_bytes, boxes of 128 bytes x box_rows, 128B swizzle
static int make_map(CUtensorMap* map, const void* base, int64_t inner, int64_t outer, int64_t ld_bytes,
                    uint32_t box_rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) {
    zib_set_error("gemm_w8a8: cuTensorMapEncodeTiled unavailable");
    return ZIB_ERR_UNSUPPORTED;
  }
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)ld_bytes};
  cuuint32_t box[2] = {(cuuint32_t)BK, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    zib_set_error("gemm_w8a8: cuTensorMapEncodeTiled failed (%d)", (int)r);
    return ZIB_ERR_INVALID_ARG;
  }
  return ZIB_OK;
}

// 0 = automatic (2-CTA pairs when M > 128), 1 = 1-CTA tiles, 2 = 2-CTA pairs
static int g_gemm_variant = 0;
constexpr int64_t kGroupBudgetDefault = 48ll << 20;
static int64_t g_group_budget = kGroupBudgetDefault;

// Blocks of the fast index per group: as few groups as keep one group's rows of the
// re-read operand within the L2 budget, of balanced sizes.
static int group_blocks(int64_t nfast, int64_t block_bytes) {
  int64_t per = g_group_budget / block_bytes;
  if (per < 1) per = 1;
  if (per >= nfast) return (int)nfast;
  const int64_t ngroups = (nfast + per - 1) / per;
  return (int)((nfast + ngroups - 1) / ngroups);
}

static int num_sms_for_current_device() {
  int dev = 0;
  cudaGetDevice(&dev);
  static int cached[64] = {0};
  if (dev < 0 || dev >= 64) return 148;
  if (!cached[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

static bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

// --- split-K tail ------------------------------------------------------------
// A launch of T tiles on C persistent CTA pairs runs ceil(T / C) waves; when the
// last wave is short (R = T mod C tiles), those R tiles are split along K into
// S = min(C / R, 4) units so that the last wave is ~1/S as long.  The partial
// int32 tiles meet in a workspace (one 128 KB slot per unit and CTA of the
// pair) with one arrival counter per tail tile and CTA; the last arrival
// resets its counter.  The caller owns the workspace: it allocates it,
// zero-fills the counters and registers it per device with
// zib_gemm_set_split_workspace (the Python layer does this with torch on first
// use); the library never allocates.  Without a registered workspace, or with
// one too small for the tail, a launch runs unsplit (or with fewer splits).
// Launches that use one workspace must not overlap on the GPU.
static bool g_split_enabled = true;
constexpr int kSplitMinKBlocks = 48;  // K >= 6144
constexpr int64_t kSplitUnitBytes = 2 * 128 * 256 * sizeof(int32_t);  // both CTAs' partial tiles
struct SplitWs {
  int32_t* ws = nullptr;
  int* ctr = nullptr;
  int units = 0;     // partial-tile pairs the workspace holds
  int tails = 0;     // tail tiles its counters cover
};
static std::mutex g_split_mu;
static SplitWs g_split_ws[64];

static SplitWs split_workspace() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return SplitWs{};
  }
  std::lock_guard<std::mutex> lk(g_split_mu);
  return g_split_ws[dev];
}

// The allocation-free variant (zib_gemm_w8a8_static_scratch), for callers that
// must not allocate device memory (a host framework that owns it through its
// own pool and budget, a stream capture in progress, a loop that cannot take
// the device synchronisation of cudaMalloc/cudaFree): the same partial slots
// and counters in static device arrays of fixed size, 64 units (16 MB) of
// partials and 128 counters, held by every GPU that loads the library.  Host
// code reaches them only through cudaGetSymbolAddress (static_scratch below);
// the counters start at zero (static initialisation) and every completed
// launch leaves them at zero.
constexpr int kStaticSplitUnits = 64;
static __device__ __align__(256) int32_t g_static_split_ws[kStaticSplitUnits * 2 * 128 * 256];
static __device__ __align__(256) int g_static_split_ctr[kStaticSplitUnits * 2];
struct StaticScratch {
  int32_t* ws = nullptr;
  int* ctr = nullptr;
};
static StaticScratch g_static_scratch[64];

// Device addresses of the static scratch on the current device, looked up once
// per device (cudaGetSymbolAddress; the first call belongs before any capture).
static int static_scratch(const StaticScratch** out, const char* what) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    zib_set_error("%s: no usable current device", what);
    return ZIB_ERR_UNSUPPORTED;
  }
  std::lock_guard<std::mutex> lk(g_split_mu);
  StaticScratch& s = g_static_scratch[dev];
  if (!s.ws) {
    void* ws = nullptr;
    void* ctr = nullptr;
    e = cudaGetSymbolAddress(&ws, g_static_split_ws);
    if (e == cudaSuccess) e = cudaGetSymbolAddress(&ctr, g_static_split_ctr);
    if (e != cudaSuccess) {
      cudaGetLastError();
      zib_set_error("%s: cudaGetSymbolAddress of the split-K scratch failed: %s", what, cudaGetErrorString(e));
      return ZIB_ERR_LAUNCH;
    }
    s.ws = static_cast<int32_t*>(ws);
    s.ctr = static_cast<int*>(ctr);
  }
  *out = &s;
  return ZIB_OK;
}

// Split of the last wave into exactly `splits` units per tile in the static
// scratch; a tail that needs more than it holds is refused before any launch.
static int plan_split_static(Params& p, int clusters, int splits, const char* what) {
  p.num_units = p.num_tiles;
  p.tail_start = p.num_tiles;
  p.splits = 1;
  const int T = p.num_tiles, C = clusters;
  if (splits <= 1 || T <= C || T % C == 0) return ZIB_OK;  // no short last wave to split
  const int R = T % C;
  ZIB_HOST_CHECK(splits <= p.num_kb, ZIB_ERR_INVALID_ARG, "%s: %d splits exceed the %d K-blocks of 128", what,
                 splits, p.num_kb);
  ZIB_HOST_CHECK(R * splits <= kStaticSplitUnits, ZIB_ERR_TOO_LARGE,
                 "%s: the last wave's %d tiles x %d splits need %d KB of split-K scratch; the static area holds "
                 "%d KB (%d units)",
                 what, R, splits, R * splits * 256, kStaticSplitUnits * 256, kStaticSplitUnits);
  const StaticScratch* sc = nullptr;
  const int st = static_scratch(&sc, what);
  if (st) return st;
  p.tail_start = T - R;
  p.splits = splits;
  p.num_units = p.tail_start + R * splits;
  p.ws = sc->ws;
  p.counters = sc->ctr;
  return ZIB_OK;
}

// Decide the split of the last wave (pair kernel, plain and int32 epilogues).
static void plan_split(Params& p, int clusters) {
  p.num_units = p.num_tiles;
  p.tail_start = p.num_tiles;
  p.splits = 1;
  const int T = p.num_tiles, C = clusters;
  // The last unit of a split tile re-reads every partial (S x 128 KB per CTA) before its
  // epilogue; that only pays off for long tiles (measured: K = 10240 gains 5%; K = 3840 loses
  // 4% at 7 waves, and 9% at 2.4 waves, where the split last wave is a larger share of the time).
  if (!g_split_enabled || T <= C || T % C == 0 || p.num_kb < kSplitMinKBlocks) return;
  const int R = T % C;
  int S = C / R;
  if (S > 4) S = 4;
  if (S > p.num_kb / 2) S = p.num_kb / 2;  // at least two K-blocks per split
  const SplitWs w = split_workspace();
  if (!w.ws || R > w.tails) return;
  if (R * S > w.units) S = w.units / R;  // as many splits as the registered workspace holds
  if (S < 2) return;
  p.tail_start = T - R;
  p.splits = S;
  p.num_units = p.tail_start + R * S;
  p.ws = w.ws;
  p.counters = w.ctr;
}

// Half units for a short last wave (pair kernel, plain and int32 epilogues,
// whole-K tiles).  R = T mod C tiles of the last wave on C CTA pairs leave
// C - R pairs idle for a whole tile; when 2R <= C they run as 2R units of 128
// output columns each, so the last wave takes about half as long (config 1,
// 1024 x 11520 x 3840: 180 tiles on 74 pairs, 2.5 tile times instead of 3).
static void plan_halves(Params& p, int clusters) {
  const int T = p.num_tiles, C = clusters;
  const int R = T % C;
  if (!g_split_enabled || R == 0 || 2 * R > C) return;
  p.tail_start = T - R;
  p.halves = 1;
  p.num_units = p.tail_start + 2 * R;
}

// M <= 8 rows: the skinny kernel (one launch, CTAs sized for four per SM).
template <int EPI>
static int launch_skinny(const void* q, int64_t ldq, const void* w, int64_t ldw, const Params& p, void* stream,
                         const char* what) {
  const int mr = p.M <= 1 ? 1 : p.M <= 2 ? 2 : p.M <= 4 ? 4 : 8;
  const size_t smem = (size_t)mr * p.K;
  const int64_t steps = ((int64_t)p.N + 7) / 8;  // warp steps of 8 columns
  int64_t grid = (steps + 7) / 8;                 // 8 warps per CTA
  const int64_t cap = (int64_t)num_sms_for_current_device() * 4;
  if (grid > cap) grid = cap;
  cudaStream_t st = (cudaStream_t)stream;
  const int8_t* qa = (const int8_t*)q;
  const int8_t* wa = (const int8_t*)w;
  switch (mr) {
    case 1: gemm_w8a8_skinny_kernel<EPI, 1><<<(unsigned)grid, 256, smem, st>>>(qa, ldq, wa, ldw, p); break;
    case 2: gemm_w8a8_skinny_kernel<EPI, 2><<<(unsigned)grid, 256, smem, st>>>(qa, ldq, wa, ldw, p); break;
    case 4: gemm_w8a8_skinny_kernel<EPI, 4><<<(unsigned)grid, 256, smem, st>>>(qa, ldq, wa, ldw, p); break;
    default: gemm_w8a8_skinny_kernel<EPI, 8><<<(unsigned)grid, 256, smem, st>>>(qa, ldq, wa, ldw, p); break;
  }
  return zib_check_launch(what);
}

// Common checks + tensor maps + launch.  w2 is the second B operand (SWIGLU: w3).
template <int EPI>
static int launch(const void* q, int64_t ldq, const void* w, const void* w2, int64_t ldw, int64_t w_rows, Params p,
                  void* stream, const char* what, int static_splits = 0) {
  const int64_t M = p.M, K = p.K;
  ZIB_HOST_CHECK(q && w && (EPI != EPI_SWIGLU || w2 || p.w13), ZIB_ERR_INVALID_ARG, "%s: null operand", what);
  ZIB_HOST_CHECK(M >= 0 && p.N > 0 && K > 0, ZIB_ERR_INVALID_ARG, "%s: bad shape M=%d N=%d K=%d", what, p.M, p.N,
                 p.K);
  ZIB_HOST_CHECK(K % 16 == 0 && ldq >= K && ldw >= K && ldq % 16 == 0 && ldw % 16 == 0, ZIB_ERR_ALIGNMENT,
                 "%s: K and row strides of q/w must be multiples of 16 (K=%lld)", what, (long long)K);
  ZIB_HOST_CHECK(aligned16(q) && aligned16(w) && (!w2 || aligned16(w2)), ZIB_ERR_ALIGNMENT,
                 "%s: q/w must be 16-byte aligned", what);
  if (M == 0) return ZIB_OK;
  if constexpr (EPI == EPI_BF16 || EPI == EPI_I32) {
    if (g_gemm_variant == 0 && M <= kSkinnyMaxM && K <= kSkinnyMaxK)
      return launch_skinny<EPI>(q, ldq, w, ldw, p, stream, what);
  }
  CUtensorMap ta, tb, tb2;
  // SWIGLU with separate w1 / w3: a 64-row box from each per CTA part; with w1 and
  // w3 as the two halves of one [2F, K] tensor: one 3-D box of 64 rows x both halves
  const bool two_b = EPI == EPI_SWIGLU && !p.w13;
  const uint32_t b_box = EPI == EPI_SWIGLU ? (uint32_t)SW_BOX_ROWS : 128u;
  int st = make_map(&ta, q, K, M, ldq, 128u);
  if (st) return st;
  if (EPI == EPI_SWIGLU && p.w13) {
    st = make_map_halves(&tb, w, K, w_rows, ldw, b_box);
    if (st) return st;
    tb2 = tb;
  } else {
    st = make_map(&tb, w, K, w_rows, ldw, b_box);
    if (st) return st;
    // plain / int32: the second map stages the 64 weight rows per CTA of a half unit
    st = make_map(&tb2, two_b ? w2 : w, K, w_rows, ldw, EPI == EPI_SWIGLU ? b_box : 64u);
    if (st) return st;
  }

  const int cols_per_tile = EPI == EPI_SWIGLU ? 128 : BN;  // output columns per tile
  p.num_nb = (p.N + cols_per_tile - 1) / cols_per_tile;
  p.num_kb = (int)((K + BK - 1) / BK);
  const int variant = g_gemm_variant;
  const bool pair = variant == 2 || (variant == 0 && M > 128);
  const int smem_bytes = pair ? Cfg<EPI>::P_SMEM : Cfg<EPI>::S_SMEM;
  static bool attr_set[2][4][64] = {{{false}}};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[pair][EPI][dev]) {
    cudaError_t e = pair ? cudaFuncSetAttribute(gemm_w8a8_pair_kernel<EPI>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes)
                         : cudaFuncSetAttribute(gemm_w8a8_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                smem_bytes);
    if (e != cudaSuccess) {
      zib_set_error("%s: cudaFuncSetAttribute failed: %s", what, cudaGetErrorString(e));
      return ZIB_ERR_LAUNCH;
    }
    attr_set[pair][EPI][dev] = true;
  }
  // The operand whose block index varies fastest is re-read by every wave of concurrent
  // tiles (it has to stay resident in L2); the other one streams once.  The smaller
  // operand takes the fast index, in groups that fit the L2 budget.
  const int64_t a_bytes = M * K, b_bytes = (int64_t)w_rows * K * (EPI == EPI_SWIGLU ? 2 : 1);
  p.n_fast = a_bytes > b_bytes ? 1 : 0;
  p.st32 = p.y && ((uintptr_t)p.y & 31) == 0 && (p.ldy & 15) == 0;
  const int sms = num_sms_for_current_device();
  if (pair) {
    p.num_mb = (int)((M + 255) / 256);
    p.num_tiles = p.num_mb * p.num_nb;
    p.group = group_blocks(p.n_fast ? p.num_nb : p.num_mb, 256 * K);  // 256 rows per block either way
    int clusters = sms / 2;
    p.num_units = p.num_tiles;
    p.tail_start = p.num_tiles;
    p.splits = 1;
    p.halves = 0;
    if (EPI == EPI_BF16 || EPI == EPI_I32) {
      if (static_splits > 0) {
        const int st = plan_split_static(p, clusters < p.num_tiles ? clusters : p.num_tiles, static_splits, what);
        if (st) return st;
      } else {
        plan_split(p, clusters);
        if (p.splits == 1) plan_halves(p, clusters);
      }
    }
    if (clusters > p.num_units) clusters = p.num_units;
    gemm_w8a8_pair_kernel<EPI><<<2 * clusters, Cfg<EPI>::THREADS, smem_bytes, (cudaStream_t)stream>>>(ta, tb, tb2, p);
  } else {
    p.num_mb = (int)((M + 127) / 128);
    p.num_tiles = p.num_mb * p.num_nb;
    p.group = group_blocks(p.n_fast ? p.num_nb : p.num_mb, (p.n_fast ? 256 : 128) * K);
    p.num_units = p.num_tiles;
    p.tail_start = p.num_tiles;
    p.splits = 1;
    int grid = sms;
    if (grid > p.num_tiles) grid = p.num_tiles;
    gemm_w8a8_kernel<EPI><<<grid, Cfg<EPI>::THREADS, smem_bytes, (cudaStream_t)stream>>>(ta, tb, tb2, p);
  }
  return zib_check_launch(what);
}

static Params base_params(int64_t M, int64_t N, int64_t K) {
  Params p{};
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  return p;
}

}  // namespace gemm
}  // namespace zib

using zib::gemm::aligned16;

extern "C" int zib_gemm_w8a8(const void* q, int64_t ldq, const void* wq, int64_t ldw, const void* sx,
                             const void* sw, const void* bias, void* y, int64_t ldy, int64_t M, int64_t N,
                             int64_t K, void* stream) {
  ZIB_HOST_CHECK(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31), ZIB_ERR_TOO_LARGE, "gemm_w8a8: too large");
  ZIB_HOST_CHECK(sx && sw && y && ldy >= N, ZIB_ERR_INVALID_ARG, "gemm_w8a8: bad epilogue operands");
  ZIB_HOST_CHECK(ldy % 8 == 0 && aligned16(y) && aligned16(sw) && (!bias || aligned16(bias)), ZIB_ERR_ALIGNMENT,
                 "gemm_w8a8: y/sw/bias must be 16-byte aligned and ldy %% 8 == 0");
  zib::gemm::Params p = zib::gemm::base_params(M, N, K);
  p.sx = (const uint16_t*)sx;
  p.sw = (const uint16_t*)sw;
  p.bias = (const uint16_t*)bias;
  p.y = (uint16_t*)y;
  p.ldy = ldy;
  return zib::gemm::launch<zib::gemm::EPI_BF16>(q, ldq, wq, nullptr, ldw, N, p, stream, "gemm_w8a8");
}

extern "C" int zib_gemm_w8a8_static_scratch(const void* q, int64_t ldq, const void* wq, int64_t ldw, const void* sx,
                                            const void* sw, const void* bias, void* y, int64_t ldy, int64_t M,
                                            int64_t N, int64_t K, int splits, void* stream) {
  ZIB_HOST_CHECK(splits >= 1 && splits <= 4, ZIB_ERR_INVALID_ARG,
                 "gemm_w8a8_static_scratch: splits must be 1 to 4 (got %d)", splits);
  ZIB_HOST_CHECK(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31), ZIB_ERR_TOO_LARGE,
                 "gemm_w8a8_static_scratch: too large");
  ZIB_HOST_CHECK(sx && sw && y && ldy >= N, ZIB_ERR_INVALID_ARG, "gemm_w8a8_static_scratch: bad epilogue operands");
  ZIB_HOST_CHECK(ldy % 8 == 0 && aligned16(y) && aligned16(sw) && (!bias || aligned16(bias)), ZIB_ERR_ALIGNMENT,
                 "gemm_w8a8_static_scratch: y/sw/bias must be 16-byte aligned and ldy %% 8 == 0");
  zib::gemm::Params p = zib::gemm::base_params(M, N, K);
  p.sx = (const uint16_t*)sx;
  p.sw = (const uint16_t*)sw;
  p.bias = (const uint16_t*)bias;
  p.y = (uint16_t*)y;
  p.ldy = ldy;
  return zib::gemm::launch<zib::gemm::EPI_BF16>(q, ldq, wq, nullptr, ldw, N, p, stream, "gemm_w8a8_static_scratch",
                                                splits);
}

extern "C" int zib_gemm_w8a8_acc_i32(const void* q, int64_t ldq, const void* wq, int64_t ldw, void* acc,
                                     int64_t ldacc, int64_t M, int64_t N, int64_t K, void* stream) {
  ZIB_HOST_CHECK(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31), ZIB_ERR_TOO_LARGE,
                 "gemm_w8a8_acc_i32: too large");
  ZIB_HOST_CHECK(acc && ldacc >= N, ZIB_ERR_INVALID_ARG, "gemm_w8a8_acc_i32: bad output");
  ZIB_HOST_CHECK(aligned16(acc), ZIB_ERR_ALIGNMENT, "gemm_w8a8_acc_i32: acc must be 16-byte aligned");
  zib::gemm::Params p = zib::gemm::base_params(M, N, K);
  p.acc = (int32_t*)acc;
  p.ldacc = ldacc;
  return zib::gemm::launch<zib::gemm::EPI_I32>(q, ldq, wq, nullptr, ldw, N, p, stream, "gemm_w8a8_acc_i32");
}

extern "C" int zib_gemm_w8a8_swiglu_had(const void* q, int64_t ldq, const void* w1, const void* w3, int64_t ldw,
                                        const void* sx, const void* sw1, const void* sw3, void* x_rot, int64_t ldo,
                                        int64_t M, int64_t F, int64_t K, void* stream) {
  ZIB_HOST_CHECK(M < (1ll << 31) && F < (1ll << 30) && K < (1ll << 31), ZIB_ERR_TOO_LARGE,
                 "gemm_w8a8_swiglu_had: too large");
  ZIB_HOST_CHECK(F > 0 && F % 128 == 0, ZIB_ERR_INVALID_ARG,
                 "gemm_w8a8_swiglu_had: features %lld not divisible by group_size 128", (long long)F);
  ZIB_HOST_CHECK(sx && sw1 && sw3 && x_rot && ldo >= F, ZIB_ERR_INVALID_ARG, "gemm_w8a8_swiglu_had: bad operands");
  ZIB_HOST_CHECK(ldo % 8 == 0 && aligned16(x_rot) && aligned16(sw1) && aligned16(sw3), ZIB_ERR_ALIGNMENT,
                 "gemm_w8a8_swiglu_had: outputs/scales must be 16-byte aligned");
  zib::gemm::Params p = zib::gemm::base_params(M, F, K);
  p.sx = (const uint16_t*)sx;
  p.sw = (const uint16_t*)sw1;
  p.sw2 = (const uint16_t*)sw3;
  p.y = (uint16_t*)x_rot;
  p.ldy = ldo;
  return zib::gemm::launch<zib::gemm::EPI_SWIGLU>(q, ldq, w1, w3, ldw, F, p, stream, "gemm_w8a8_swiglu_had");
}

namespace zib {
namespace gemm {

// One [2F, K] int8 weight of alternating 32-row blocks (w1 rows 32g..32g+31,
// then w3 rows 32g..32g+31, g = 0 .. F/32-1) from w1 and w3 [F, K] (row
// stride ldw): each thread moves 16 bytes.
}  // namespace gemm
}  // namespace zib

extern "C" int zib_gemm_w8a8_swiglu_had_w13(const void* q, int64_t ldq, const void* w13, int64_t ldw,
                                            const void* sx, const void* sw1, const void* sw3, void* x_rot,
                                            int64_t ldo, int64_t M, int64_t F, int64_t K, void* stream) {
  ZIB_HOST_CHECK(M < (1ll << 31) && F < (1ll << 30) && K < (1ll << 31), ZIB_ERR_TOO_LARGE,
                 "gemm_w8a8_swiglu_had_w13: too large");
  ZIB_HOST_CHECK(F > 0 && F % 128 == 0, ZIB_ERR_INVALID_ARG,
                 "gemm_w8a8_swiglu_had_w13: features %lld not divisible by group_size 128", (long long)F);
  ZIB_HOST_CHECK(sx && sw1 && sw3 && x_rot && ldo >= F, ZIB_ERR_INVALID_ARG,
                 "gemm_w8a8_swiglu_had_w13: bad operands");
  ZIB_HOST_CHECK(ldo % 8 == 0 && aligned16(x_rot) && aligned16(sw1) && aligned16(sw3), ZIB_ERR_ALIGNMENT,
                 "gemm_w8a8_swiglu_had_w13: outputs/scales must be 16-byte aligned");
  zib::gemm::Params p = zib::gemm::base_params(M, F, K);
  p.sx = (const uint16_t*)sx;
  p.sw = (const uint16_t*)sw1;
  p.sw2 = (const uint16_t*)sw3;
  p.y = (uint16_t*)x_rot;
  p.ldy = ldo;
  p.w13 = 1;
  return zib::gemm::launch<zib::gemm::EPI_SWIGLU>(q, ldq, w13, nullptr, ldw, F, p, stream,
                                                   "gemm_w8a8_swiglu_had_w13");
}

extern "C" int zib_gemm_w8a8_qk_norm_rope(const void* q, int64_t ldq, const void* wq, int64_t ldw, const void* sx,
                                          const void* sw, void* y, int64_t ldy, int64_t M, int64_t N, int64_t K,
                                          const float* q_norm_w, const float* k_norm_w, float q_eps, float k_eps,
                                          const float* cosp, const float* sinp, int64_t cs_b, int64_t seq,
                                          int64_t heads, void* stream) {
  ZIB_HOST_CHECK(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31), ZIB_ERR_TOO_LARGE,
                 "gemm_w8a8_qk_norm_rope: too large");
  ZIB_HOST_CHECK(heads > 0 && heads % 2 == 0 && N == 3 * heads * 128 && seq > 0 && M % seq == 0,
                 ZIB_ERR_INVALID_ARG,
                 "gemm_w8a8_qk_norm_rope: needs N = 3*heads*128 with an even head count and M a multiple of seq");
  ZIB_HOST_CHECK(cs_b >= 0 && (M / seq) * cs_b + seq * 64 < (1ll << 31), ZIB_ERR_TOO_LARGE,
                 "gemm_w8a8_qk_norm_rope: cos/sin tables beyond 2^31 elements");
  ZIB_HOST_CHECK(sx && sw && y && ldy >= N && q_norm_w && k_norm_w && cosp && sinp, ZIB_ERR_INVALID_ARG,
                 "gemm_w8a8_qk_norm_rope: bad operands");
  ZIB_HOST_CHECK(ldy % 8 == 0 && aligned16(y) && aligned16(sw) && aligned16(q_norm_w) && aligned16(k_norm_w) &&
                     aligned16(cosp) && aligned16(sinp) && cs_b % 4 == 0,
                 ZIB_ERR_ALIGNMENT, "gemm_w8a8_qk_norm_rope: operands must be 16-byte aligned");
  zib::gemm::Params p = zib::gemm::base_params(M, N, K);
  p.sx = (const uint16_t*)sx;
  p.sw = (const uint16_t*)sw;
  p.y = (uint16_t*)y;
  p.ldy = ldy;
  p.qn_w = q_norm_w;
  p.kn_w = k_norm_w;
  p.q_eps = q_eps;
  p.k_eps = k_eps;
  p.cosp = cosp;
  p.sinp = sinp;
  p.cs_b = cs_b;
  p.seq = (int)seq;
  p.heads = (int)heads;
  return zib::gemm::launch<zib::gemm::EPI_QKROPE>(q, ldq, wq, nullptr, ldw, N, p, stream, "gemm_w8a8_qk_norm_rope");
}

// Self-test of the bounded-wait path: one thread waits on an mbarrier that
// nothing arrives at, so the wait gives up after its limit (2 s), records
// ZIB_ERR_TIMEOUT in the device error word and returns; nothing faults, traps
// or hangs, and the context stays usable.
__global__ void selftest_wait_kernel() {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    zib::mbar_init(&bar, 1);
    abort_flag = 0;
    zib::mbar_fence_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) (void)zib::mbar_wait_bounded(&bar, 0, &abort_flag);
}

extern "C" int zib_selftest_bounded_wait(void* stream) {
  selftest_wait_kernel<<<1, 32, 0, (cudaStream_t)stream>>>();
  return zib_check_launch("selftest_bounded_wait");
}

extern "C" int zib_gemm_set_split_workspace(int device, void* ws, int64_t ws_bytes, void* counters,
                                            int64_t n_counters) {
  ZIB_HOST_CHECK(device >= 0 && device < 64, ZIB_ERR_INVALID_ARG, "gemm_set_split_workspace: bad device %d",
                 device);
  ZIB_HOST_CHECK((ws == nullptr) == (counters == nullptr), ZIB_ERR_INVALID_ARG,
                 "gemm_set_split_workspace: register both buffers or neither");
  ZIB_HOST_CHECK(!ws || (ws_bytes >= zib::gemm::kSplitUnitBytes && n_counters >= 2), ZIB_ERR_INVALID_ARG,
                 "gemm_set_split_workspace: needs at least %lld bytes and 2 counters",
                 (long long)zib::gemm::kSplitUnitBytes);
  ZIB_HOST_CHECK(!ws || (((uintptr_t)ws & 15) == 0 && ((uintptr_t)counters & 3) == 0), ZIB_ERR_ALIGNMENT,
                 "gemm_set_split_workspace: the workspace must be 16-byte aligned");
  std::lock_guard<std::mutex> lk(zib::gemm::g_split_mu);
  zib::gemm::SplitWs& w = zib::gemm::g_split_ws[device];
  w.ws = static_cast<int32_t*>(ws);
  w.ctr = static_cast<int*>(counters);
  const int64_t units = ws ? ws_bytes / zib::gemm::kSplitUnitBytes : 0;
  w.units = (int)(units < (1 << 20) ? units : (1 << 20));
  w.tails = ws ? (int)((n_counters / 2) < (1 << 20) ? n_counters / 2 : (1 << 20)) : 0;
  return ZIB_OK;
}

extern "C" int zib_gemm_set_split(int enable) {
  zib::gemm::g_split_enabled = enable != 0;
  return ZIB_OK;
}

// zero every split-K arrival counter (after a device error left a launch unfinished)
void zib_gemm_split_reset() {
  std::lock_guard<std::mutex> lk(zib::gemm::g_split_mu);
  int dev = 0;
  cudaGetDevice(&dev);
  for (int d = 0; d < 64; ++d) {
    zib::gemm::SplitWs& w = zib::gemm::g_split_ws[d];
    zib::gemm::StaticScratch& sc = zib::gemm::g_static_scratch[d];
    if (!w.ctr && !sc.ctr) continue;
    cudaSetDevice(d);
    cudaDeviceSynchronize();  // no GEMM of this device is still counting on any stream
    if (w.ctr) cudaMemset(w.ctr, 0, (size_t)w.tails * 2 * sizeof(int));
    if (sc.ctr) cudaMemset(sc.ctr, 0, sizeof(zib::gemm::g_static_split_ctr));
    cudaDeviceSynchronize();
  }
  cudaSetDevice(dev);
  cudaGetLastError();
}

extern "C" int zib_gemm_set_group_budget(int64_t bytes) {
  if (bytes < 0) {
    zib_set_error("gemm_set_group_budget: bytes must be >= 0");
    return ZIB_ERR_INVALID_ARG;
  }
  zib::gemm::g_group_budget = bytes > 0 ? bytes : zib::gemm::kGroupBudgetDefault;
  return ZIB_OK;
}

extern "C" int zib_gemm_set_variant(int variant) {
  if (variant < 0 || variant > 2) {
    zib_set_error("gemm_set_variant: variant must be 0, 1 or 2");
    return ZIB_ERR_INVALID_ARG;
  }
  zib::gemm::g_gemm_variant = variant;
  return ZIB_OK;
}
