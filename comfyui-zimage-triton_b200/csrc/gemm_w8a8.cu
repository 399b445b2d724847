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
//   warps 2..5  epilogue: tcgen05.ld 32x32b of the finished accumulator,
//               dequant + bias + bf16 rounding in registers, global stores;
//               overlaps the next tile's MMAs (double-buffered TMEM).
// Every mbarrier wait is bounded (globaltimer); on expiry the CTA records
// ZIB_ERR_TIMEOUT in a device error word, drains its in-flight TMA loads and
// MMAs, frees TMEM and exits.  No TMA multicast is used anywhere.
#include "zib_common.cuh"

#include <cuda.h>
#include <mutex>

__device__ int g_zib_device_error = 0;

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
constexpr int NUM_THREADS = 192;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align slack*/ + 256 /*barriers*/;
constexpr unsigned long long kTimeoutNs = 2000000000ull;  // 2 s per wait

// instruction descriptor: D=s32, A=B=s8, both K-major, N=256, M=128
constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                            ((uint32_t)(BM >> 4) << 24);

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: returns false (and raises the CTA abort flag) after kTimeoutNs,
// or as soon as another role has raised the abort flag.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer() - t0 > kTimeoutNs) {
      *abort_flag = 1;
      atomicExch(&g_zib_device_error, (int)ZIB_ERR_TIMEOUT);
      return false;
    }
  }
}

// Wait used while draining after an abort: bounded, never raises the flag.
__device__ __forceinline__ void mbar_drain_wait(uint64_t* bar, uint32_t parity) {
  const unsigned long long t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > kTimeoutNs) return;
  }
}

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
      mbar_init(&tempty_bar[a], 4);
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
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag)) { ok = false; break; }
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
        if (!mbar_wait(&tempty_bar[accb], acc_phase ^ 1u, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(accb * BN);
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, abort_flag)) { ok = false; break; }
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
    // ---------------- epilogue (warps 2..5) ----------------
    const int quarter = warp & 3;  // TMEM lanes [32*quarter, 32*quarter+32)
    int accb = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
      int ok = 1;
      if (lane == 0) ok = mbar_wait(&tfull_bar[accb], acc_phase, abort_flag) ? 1 : 0;
      ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      const int mb = tile % p.num_mb, nb = tile / p.num_mb;
      const int row = mb * BM + quarter * 32 + lane;
      const bool row_ok = row < p.M;
      float sxf = 0.0f;
      if (!ACC_OUT && row_ok) sxf = bf16_bits_to_float(p.sx[row]);
      const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(accb * BN);
#pragma unroll 1
      for (int ch = 0; ch < BN / 32; ++ch) {
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
              const float s = bf16_round(__fmul_rn(sxf, swv[t]));
              const float a = bf16_round(__int2float_rn((int)r[j + t]));
              float v = bf16_round(__fmul_rn(a, s));
              if (p.bias) v = bf16_round(__fadd_rn(v, bv[t]));
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

  static bool attr_set[2][64] = {{false}};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[ACC_OUT][dev]) {
    cudaError_t e = cudaFuncSetAttribute(gemm_w8a8_kernel<ACC_OUT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         SMEM_BYTES);
    if (e != cudaSuccess) {
      zib_set_error("gemm_w8a8: cudaFuncSetAttribute failed: %s", cudaGetErrorString(e));
      return ZIB_ERR_LAUNCH;
    }
    attr_set[ACC_OUT][dev] = true;
  }
  int grid = num_sms_for_current_device();
  if (grid > p.num_tiles) grid = p.num_tiles;
  gemm_w8a8_kernel<ACC_OUT><<<grid, NUM_THREADS, SMEM_BYTES, (cudaStream_t)stream>>>(ta, tb, p);
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

extern "C" int zib_device_error_read_clear(void) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_zib_device_error, sizeof(int)) != cudaSuccess) return ZIB_ERR_LAUNCH;
  int zero = 0;
  cudaMemcpyToSymbol(g_zib_device_error, &zero, sizeof(int));
  return v;
}
