// K1: W8A8 GEMM on 5th-generation tensor cores (tcgen05, kind::i8) for sm_100a.
//
// Replaces torch._int_mm plus the eager dequant epilogue of the reference's
// W8A8+Hadamard linear (src/zimage_triton/quantization/int8_linear.py:133-137):
//   acc[m,n] = sum_k q[m,k] * wq[n,k]                         (int32, exact)
//   y[m,n]   = bf16( bf16(acc) * bf16(sx[m] * sw[n]) ) (+ bias[n])
//
// Design (one CTA per SM, persistent over 128x256 output tiles):
//   warp 0      TMA producer: 128x128 A tile + 256x128 B tile per k-block,
//               128-byte swizzle, 4-stage shared-memory ring.
//   warp 1      owns TMEM (512 columns = two 128x256 int32 accumulators) and
//               issues tcgen05.mma (M=128, N=256, K=32) from one thread.
//   warps 2..9  epilogue (two warps per TMEM lane quarter, 128 columns each):
//               tcgen05.ld 32x32b of the finished accumulator,
//               dequant + bias + bf16 rounding in registers, global stores;
//               overlaps the next tile's MMAs (double-buffered TMEM).
// Every mbarrier wait is bounded (globaltimer); on expiry the CTA records
// ZIB_ERR_TIMEOUT in a device error word, drains its in-flight TMA loads and
// MMAs, frees TMEM and exits.  No TMA multicast is used anywhere.
#include "zib_async.cuh"

#include <cuda.h>
#include <mutex>

ZIB_DEFINE_ERROR_READER(zib_err_read_clear_gemm)

namespace zib {
namespace gemm {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 128;  // bytes == int8 elements == one 128-byte swizzle row
constexpr int STAGES = 4;
constexpr int UMMA_K = 32;
constexpr int A_BYTES = BM * BK;
constexpr int B_BYTES = BN * BK;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int TMEM_COLS = 512;
constexpr int NUM_THREADS = 320;  // warp 0 TMA, warp 1 MMA/TMEM, warps 2..9 epilogue
constexpr int EPI_WARPS = 8;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align slack*/ + 256 /*barriers*/;

// instruction descriptor: D=s32, A=B=s8, both K-major, N=256, M=128
constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                            ((uint32_t)(BM >> 4) << 24);

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// K-major operand tile in shared memory written by TMA with 128-byte swizzle:
// rows of 128 bytes, 8-row core groups 1024 bytes apart (SBO), version 1.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;           // leading byte offset (unused with 128B swizzle)
  d |= (uint64_t)(1024u >> 4) << 32; // stride byte offset
  d |= (uint64_t)1u << 46;           // descriptor version for tcgen05
  d |= (uint64_t)2u << 61;           // SWIZZLE_128B
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

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
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

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

struct Params {
  int M, N, K;
  int num_mb, num_nb, num_kb, num_tiles;
  const uint16_t* sx;
  const uint16_t* sw;
  const uint16_t* bias;
  uint16_t* y;
  int64_t ldy;
  int32_t* acc;
  int64_t ldacc;
};

// Dequant epilogue of one thread's accumulator row (128-row x 256-column tile
// in TMEM, this thread = one row): tcgen05.ld 32 columns at a time, then
// y = bf16(bf16(acc) * bf16(sx*sw)) (+ bias), or the raw int32 accumulators.
// bf16 round-to-nearest-even on the ALU pipe (finite inputs); keeps the
// conversion (XU) pipe for the int32 -> fp32 conversions.
__device__ __forceinline__ float bf16_rne_alu(float v) {
  uint32_t b = __float_as_uint(v);
  b += 0x7FFFu + ((b >> 16) & 1u);
  return __uint_as_float(b & 0xFFFF0000u);
}

template <bool ACC_OUT>
__device__ __forceinline__ void epilogue_rows(const Params& p, uint32_t t_row, int row, int nb, int ch_begin,
                                              int ch_end) {
  const bool row_ok = row < p.M;
  float sxf = 0.0f;
  if (!ACC_OUT && row_ok) sxf = bf16_bits_to_float(p.sx[row]);
#pragma unroll 1
  for (int ch = ch_begin; ch < ch_end; ++ch) {
    uint32_t r[32];
    __syncwarp();  // tcgen05.ld is .sync.aligned: the whole warp issues it converged
    tmem_ld32(t_row + (uint32_t)(ch * 32), r);
    tmem_wait_ld();
    const int n0 = nb * BN + ch * 32;
    if (!row_ok || n0 >= p.N) continue;
    const bool full = n0 + 32 <= p.N;
    if (ACC_OUT) {
      int32_t* dst = p.acc + (int64_t)row * p.ldacc + n0;
      if (full && (p.ldacc % 4) == 0) {
#pragma unroll
        for (int j = 0; j < 32; j += 4)
          *reinterpret_cast<int4*>(dst + j) = make_int4((int)r[j], (int)r[j + 1], (int)r[j + 2], (int)r[j + 3]);
      } else {
        for (int j = 0; j < 32 && n0 + j < p.N; ++j) dst[j] = (int)r[j];
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
          const float s = bf16_rne_alu(__fmul_rn(sxf, swv[t]));
          const float a = bf16_rne_alu(__int2float_rn((int)r[j + t]));
          float v = bf16_rne_alu(__fmul_rn(a, s));
          if (p.bias) v = bf16_rne_alu(__fadd_rn(v, bv[t]));
          out[j + t] = v;
        }
      }
      uint16_t* dst = p.y + (int64_t)row * p.ldy + n0;
      if (full) {
#pragma unroll
        for (int j = 0; j < 32; j += 8) store_bf16x8(dst + j, out + j);
      } else {
        for (int j = 0; j < 32 && n0 + j < p.N; ++j) dst[j] = (uint16_t)(__float_as_uint(out[j]) >> 16);
      }
    }
  }
}

template <bool ACC_OUT>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_w8a8_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                     const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smem_a = smem;                          // STAGES x A_BYTES
  uint8_t* smem_b = smem + STAGES * A_BYTES;       // STAGES x B_BYTES
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* full_bar = bars;                       // [STAGES]
  uint64_t* empty_bar = bars + STAGES;             // [STAGES]
  uint64_t* tfull_bar = bars + 2 * STAGES;         // [2]
  uint64_t* tempty_bar = bars + 2 * STAGES + 2;    // [2]
  uint64_t* mma_done_bar = bars + 2 * STAGES + 4;  // [1]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], EPI_WARPS);
    }
    mbar_init(mma_done_bar, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
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
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t pend_mask = 0, pend_parity = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        const int mb = tile % p.num_mb, nb = tile / p.num_mb;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait_bounded(&empty_bar[stage], phase ^ 1u, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&full_bar[stage], STAGE_BYTES);
          tma_load_2d(smem_a + stage * A_BYTES, &tmap_a, &full_bar[stage], kb * BK, mb * BM);
          tma_load_2d(smem_b + stage * B_BYTES, &tmap_b, &full_bar[stage], kb * BK, nb * BN);
          pend_mask |= 1u << stage;
          pend_parity = (pend_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      if (!ok) {
        // drain: every stage has at most one load in flight; wait for it to land
        for (int s = 0; s < STAGES; ++s)
          if (pend_mask & (1u << s)) mbar_drain_wait(&full_bar[s], (pend_parity >> s) & 1u);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int accb = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      const uint32_t a_base = smem_u32(smem_a), b_base = smem_u32(smem_b);
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        if (!mbar_wait_bounded(&tempty_bar[accb], acc_phase ^ 1u, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(accb * BN);
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait_bounded(&full_bar[stage], phase, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint64_t adesc = sdesc_sw128(a_base + stage * A_BYTES);
          const uint64_t bdesc = sdesc_sw128(b_base + stage * B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / UMMA_K; ++k) {
            // advance the start address by k*32 bytes inside the swizzle atom
            umma_i8(d_tmem, adesc + (uint64_t)((k * UMMA_K) >> 4), bdesc + (uint64_t)((k * UMMA_K) >> 4), kIdesc,
                    (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(&empty_bar[stage]);  // frees the smem stage once these MMAs retire
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        umma_commit(&tfull_bar[accb]);
        accb ^= 1;
        if (accb == 0) acc_phase ^= 1u;
      }
      // all MMAs issued by this thread retire before TMEM is released
      umma_commit(mma_done_bar);
      mbar_drain_wait(mma_done_bar, 0);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue (warps 2..9) ----------------
    // warp w reads TMEM lanes [32*(w%4), +32); warps w and w+4 split the 256 columns
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    int accb = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
      int ok = 1;
      if (lane == 0) ok = mbar_wait_bounded(&tfull_bar[accb], acc_phase, abort_flag) ? 1 : 0;
      ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      const int mb = tile % p.num_mb, nb = tile / p.num_mb;
      epilogue_rows<ACC_OUT>(p, tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(accb * BN),
                             mb * BM + quarter * 32 + lane, nb, half * 4, half * 4 + 4);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty_bar[accb]);
      accb ^= 1;
      if (accb == 0) acc_phase ^= 1u;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                 : "memory");
  }
}

// ---------------------------------------------------------------------------
// 2-CTA variant (cta_group::2).  A cluster of two CTAs on two SMs computes a
// 256x256 output tile: each CTA stages its own 128 rows of A and 128 of the
// tile's 256 B rows (32 KB per 128-deep k-block, 6 stages), both CTAs' TMA
// loads complete on the leader's full barrier, the leader CTA issues
// M=256 x N=256 x K=32 MMAs that read both CTAs' shared memory, and each CTA's
// TMEM receives its 128 accumulator rows.  Per SM this halves the B traffic
// through shared memory relative to the 1-CTA 128x256 tile.  TMA loads carry
// .cta_group::2 only; no load uses cluster multicast.  The leader's MMA
// commits are multicast to both CTAs' barriers (tcgen05.commit), and both
// CTAs' epilogue warps release an accumulator on the leader's barrier.
// ---------------------------------------------------------------------------
constexpr int P_STAGES = 6;
constexpr int P_A_BYTES = 128 * BK;
constexpr int P_B_BYTES = 128 * BK;
constexpr int P_STAGE_BYTES = P_A_BYTES + P_B_BYTES;
constexpr int P_SMEM_BYTES = P_STAGES * P_STAGE_BYTES + 1024 + 256;
// D=s32, A=B=s8, K-major, N=256, M=256
constexpr uint32_t kIdescPair = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(256 >> 3) << 17) |
                                ((uint32_t)(256 >> 4) << 24);

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

__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t mbar_cluster, int x,
                                                 int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
      "%4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(mbar_cluster), "r"(x), "r"(y)
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

// Arrive (when all prior MMAs of this thread retire) on `bar` in every CTA of `mask`.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar, uint16_t mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(mask)
      : "memory");
}

template <bool ACC_OUT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
    gemm_w8a8_pair_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                          const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem + P_STAGES * P_A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + P_STAGES * P_STAGE_BYTES);
  uint64_t* full_bar = bars;                          // [P_STAGES]  (leader's is used)
  uint64_t* empty_bar = bars + P_STAGES;              // [P_STAGES]  (both)
  uint64_t* tfull_bar = bars + 2 * P_STAGES;          // [2]         (both)
  uint64_t* tempty_bar = bars + 2 * P_STAGES + 2;     // [2]         (leader's is used)
  uint64_t* mma_done_bar = bars + 2 * P_STAGES + 4;   // [1]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 2 * P_STAGES + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int cluster_id = blockIdx.x >> 1;
  const int nclusters = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 2 * EPI_WARPS);  // epilogue warps of both CTAs
    }
    mbar_init(mma_done_bar, 1);
    *abort_flag = 0;
    mbar_fence_init();
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
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
    // ---------------- TMA producer (both CTAs) ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t pend_mask = 0, pend_parity = 0;
      bool ok = true;
      for (int tile = cluster_id; tile < p.num_tiles && ok; tile += nclusters) {
        const int mb = tile % p.num_mb, nb = tile / p.num_mb;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait_bounded(&empty_bar[stage], phase ^ 1u, abort_flag)) { ok = false; break; }
          const uint32_t fb = smem_u32(&full_bar[stage]);
          if (leader) mbar_arrive_expect_tx(&full_bar[stage], 2 * P_STAGE_BYTES);
          const uint32_t fb_leader = leader ? fb : mapa_rank(fb, 0);
          tma_load_2d_pair(smem_a + stage * P_A_BYTES, &tmap_a, fb_leader, kb * BK, mb * 256 + (int)rank * 128);
          tma_load_2d_pair(smem_b + stage * P_B_BYTES, &tmap_b, fb_leader, kb * BK, nb * 256 + (int)rank * 128);
          pend_mask |= 1u << stage;
          pend_parity = (pend_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == P_STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      if (!ok) {
        aborted = true;
        if (leader) {
          for (int s = 0; s < P_STAGES; ++s)
            if (pend_mask & (1u << s)) mbar_drain_wait(&full_bar[s], (pend_parity >> s) & 1u);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader CTA only) ----------------
    if (lane == 0 && leader) {
      int stage = 0;
      uint32_t phase = 0;
      int accb = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      const uint32_t a_base = smem_u32(smem_a), b_base = smem_u32(smem_b);
      for (int tile = cluster_id; tile < p.num_tiles && ok; tile += nclusters) {
        if (!mbar_wait_bounded(&tempty_bar[accb], acc_phase ^ 1u, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(accb * BN);
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait_bounded(&full_bar[stage], phase, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint64_t adesc = sdesc_sw128(a_base + stage * P_A_BYTES);
          const uint64_t bdesc = sdesc_sw128(b_base + stage * P_B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / UMMA_K; ++k) {
            umma_i8_pair(d_tmem, adesc + (uint64_t)((k * UMMA_K) >> 4), bdesc + (uint64_t)((k * UMMA_K) >> 4),
                         kIdescPair, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit_pair(&empty_bar[stage], (uint16_t)3);  // frees the stage in both CTAs
          if (++stage == P_STAGES) { stage = 0; phase ^= 1u; }
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
    // ---------------- epilogue (warps 2..9, both CTAs) ----------------
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    int accb = 0;
    uint32_t acc_phase = 0;
    const uint32_t tempty_leader0 = mapa_rank(smem_u32(&tempty_bar[0]), 0);
    for (int tile = cluster_id; tile < p.num_tiles; tile += nclusters) {
      int ok = 1;
      if (lane == 0) ok = mbar_wait_bounded(&tfull_bar[accb], acc_phase, abort_flag) ? 1 : 0;
      ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
      if (!ok) { aborted = true; break; }
      tc_fence_after();
      const int mb = tile % p.num_mb, nb = tile / p.num_mb;
      epilogue_rows<ACC_OUT>(p, tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(accb * BN),
                             mb * 256 + (int)rank * 128 + quarter * 32 + lane, nb, half * 4, half * 4 + 4);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_leader0 + (uint32_t)(accb * 8));
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
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                 : "memory");
  }
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

static int make_map(CUtensorMap* map, const void* base, int64_t inner, int64_t outer, int64_t ld_bytes,
                    int box_inner, int box_outer) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) {
    zib_set_error("gemm_w8a8: cuTensorMapEncodeTiled unavailable");
    return ZIB_ERR_UNSUPPORTED;
  }
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)ld_bytes};
  cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_outer};
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

template <bool ACC_OUT>
static int launch(const void* q, int64_t ldq, const void* wq, int64_t ldw, const void* sx, const void* sw,
                  const void* bias, void* y, int64_t ldy, void* acc, int64_t ldacc, int64_t M, int64_t N, int64_t K,
                  void* stream) {
  ZIB_HOST_CHECK(q && wq, ZIB_ERR_INVALID_ARG, "gemm_w8a8: null operand");
  ZIB_HOST_CHECK(M >= 0 && N > 0 && K > 0, ZIB_ERR_INVALID_ARG, "gemm_w8a8: bad shape M=%lld N=%lld K=%lld",
                 (long long)M, (long long)N, (long long)K);
  ZIB_HOST_CHECK(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31), ZIB_ERR_TOO_LARGE, "gemm_w8a8: too large");
  ZIB_HOST_CHECK(K % 16 == 0 && ldq >= K && ldw >= K && ldq % 16 == 0 && ldw % 16 == 0, ZIB_ERR_ALIGNMENT,
                 "gemm_w8a8: K and row strides of q/wq must be multiples of 16 (K=%lld)", (long long)K);
  ZIB_HOST_CHECK(((uintptr_t)q & 15) == 0 && ((uintptr_t)wq & 15) == 0, ZIB_ERR_ALIGNMENT,
                 "gemm_w8a8: q/wq must be 16-byte aligned");
  if (ACC_OUT) {
    ZIB_HOST_CHECK(acc && ldacc >= N, ZIB_ERR_INVALID_ARG, "gemm_w8a8_acc_i32: bad output");
    ZIB_HOST_CHECK(((uintptr_t)acc & 15) == 0, ZIB_ERR_ALIGNMENT, "gemm_w8a8_acc_i32: acc must be 16-byte aligned");
  } else {
    ZIB_HOST_CHECK(sx && sw && y && ldy >= N, ZIB_ERR_INVALID_ARG, "gemm_w8a8: bad epilogue operands");
    ZIB_HOST_CHECK(ldy % 8 == 0 && ((uintptr_t)y & 15) == 0 && ((uintptr_t)sw & 15) == 0 &&
                       (!bias || ((uintptr_t)bias & 15) == 0),
                   ZIB_ERR_ALIGNMENT, "gemm_w8a8: y/sw/bias must be 16-byte aligned and ldy %% 8 == 0");
  }
  if (M == 0) return ZIB_OK;
  CUtensorMap ta, tb;
  int st = make_map(&ta, q, K, M, ldq, BK, BM);
  if (st) return st;
  st = make_map(&tb, wq, K, N, ldw, BK, BN);
  if (st) return st;

  Params p;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.num_mb = (int)((M + BM - 1) / BM);
  p.num_nb = (int)((N + BN - 1) / BN);
  p.num_kb = (int)((K + BK - 1) / BK);
  p.num_tiles = p.num_mb * p.num_nb;
  p.sx = (const uint16_t*)sx;
  p.sw = (const uint16_t*)sw;
  p.bias = (const uint16_t*)bias;
  p.y = (uint16_t*)y;
  p.ldy = ldy;
  p.acc = (int32_t*)acc;
  p.ldacc = ldacc;

  const int variant = g_gemm_variant;
  const bool pair = variant == 2 || (variant == 0 && M > 128);
  static bool attr_set[2][2][64] = {{{false}}};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[pair][ACC_OUT][dev]) {
    cudaError_t e = pair ? cudaFuncSetAttribute(gemm_w8a8_pair_kernel<ACC_OUT>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize, P_SMEM_BYTES)
                         : cudaFuncSetAttribute(gemm_w8a8_kernel<ACC_OUT>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) {
      zib_set_error("gemm_w8a8: cudaFuncSetAttribute failed: %s", cudaGetErrorString(e));
      return ZIB_ERR_LAUNCH;
    }
    attr_set[pair][ACC_OUT][dev] = true;
  }
  const int sms = num_sms_for_current_device();
  if (pair) {
    // B tiles are re-described with 128-row boxes (each CTA stages half of the 256-row tile)
    st = make_map(&tb, wq, K, N, ldw, BK, 128);
    if (st) return st;
    p.num_mb = (int)((M + 255) / 256);
    p.num_tiles = p.num_mb * p.num_nb;
    int clusters = sms / 2;
    if (clusters > p.num_tiles) clusters = p.num_tiles;
    gemm_w8a8_pair_kernel<ACC_OUT><<<2 * clusters, NUM_THREADS, P_SMEM_BYTES, (cudaStream_t)stream>>>(ta, tb, p);
  } else {
    int grid = sms;
    if (grid > p.num_tiles) grid = p.num_tiles;
    gemm_w8a8_kernel<ACC_OUT><<<grid, NUM_THREADS, SMEM_BYTES, (cudaStream_t)stream>>>(ta, tb, p);
  }
  return zib_check_launch(ACC_OUT ? "gemm_w8a8_acc_i32" : "gemm_w8a8");
}

}  // namespace gemm
}  // namespace zib

extern "C" int zib_gemm_w8a8(const void* q, int64_t ldq, const void* wq, int64_t ldw, const void* sx,
                             const void* sw, const void* bias, void* y, int64_t ldy, int64_t M, int64_t N,
                             int64_t K, void* stream) {
  return zib::gemm::launch<false>(q, ldq, wq, ldw, sx, sw, bias, y, ldy, nullptr, 0, M, N, K, stream);
}

extern "C" int zib_gemm_w8a8_acc_i32(const void* q, int64_t ldq, const void* wq, int64_t ldw, void* acc,
                                     int64_t ldacc, int64_t M, int64_t N, int64_t K, void* stream) {
  return zib::gemm::launch<true>(q, ldq, wq, ldw, nullptr, nullptr, nullptr, nullptr, 0, acc, ldacc, M, N, K,
                                 stream);
}

extern "C" int zib_gemm_set_variant(int variant) {
  if (variant < 0 || variant > 2) {
    zib_set_error("gemm_set_variant: variant must be 0, 1 or 2");
    return ZIB_ERR_INVALID_ARG;
  }
  zib::gemm::g_gemm_variant = variant;
  return ZIB_OK;
}
