/*
 * zimage_b200.h - C ABI of libzimage_b200.so, the sm_100a (B200) kernels of
 * the Z-Image S3-DiT W8A8 forward path.
 *
 * Conventions for every entry point:
 *   - Plain device pointers, element counts and row strides (in ELEMENTS);
 *     no framework types.  `stream` is a cudaStream_t passed as void*.
 *   - The caller allocates every output.  Kernels never allocate, free or
 *     synchronise; work is enqueued on `stream`.
 *   - Return 0 (ZIB_OK) or a zib_status code; zib_last_error() gives a
 *     thread-local message.  Shape/dtype/alignment problems are detected on
 *     the host before any launch (the Python layer maps them to ValueError /
 *     RuntimeError like the reference: kernels/swiglu.py:82-86,
 *     kernels/utils.py:33-37).
 *   - bf16 tensors are raw uint16 bf16 bit patterns; "f32" tensors are float.
 *
 * Each declaration names the reference interface it replaces (file:line
 * within newgrit1004/ComfyUI-ZImage-Triton).
 */
#ifndef ZIMAGE_B200_H_
#define ZIMAGE_B200_H_

#include <stdint.h>

#if defined(__GNUC__)
#define ZIB_API __attribute__((visibility("default")))
#else
#define ZIB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum zib_status {
  ZIB_OK = 0,
  ZIB_ERR_INVALID_ARG = 1, /* bad shape / null pointer       -> ValueError   */
  ZIB_ERR_ALIGNMENT = 2,   /* pointer or stride misaligned   -> ValueError   */
  ZIB_ERR_UNSUPPORTED = 3, /* no sm_100 device / feature     -> RuntimeError */
  ZIB_ERR_LAUNCH = 4,      /* CUDA launch/driver error       -> RuntimeError */
  ZIB_ERR_TOO_LARGE = 5,   /* row longer than supported      -> RuntimeError */
  ZIB_ERR_TIMEOUT = 6      /* a bounded device wait expired  -> RuntimeError */
} zib_status;

/* Library version (major*10000 + minor*100 + patch). */
ZIB_API int zib_version(void);
/* Human-readable text of a zib_status. */
ZIB_API const char* zib_status_string(int status);
/* Message of the last failing call on this host thread ("" if none). */
ZIB_API const char* zib_last_error(void);
/* 0 if device `dev` is an sm_100 part this library can run on, else a zib_status. */
ZIB_API int zib_device_check(int dev);
/* Reads and clears the device-side error word of the current device (set by a
 * kernel whose bounded wait expired: ZIB_ERR_TIMEOUT).  Synchronises the current
 * device first (every stream, non-blocking ones included) and, after a GEMM
 * error, each device whose split-K counters it re-zeroes; not for the hot path
 * nor inside a stream capture.  Returns 0 when no kernel reported an error. */
ZIB_API int zib_device_error_read_clear(void);
/* Launches one thread that waits on a barrier nothing arrives at: the bounded
 * wait of the GEMM and row kernels expires (2 s), the device error word reads
 * ZIB_ERR_TIMEOUT afterwards, and the context stays usable.  Exercises the
 * failure path without a fault.  No counterpart in the reference. */
ZIB_API int zib_selftest_bounded_wait(void* stream);

/* ---------------------------------------------------------------------------
 * W8A8 + Hadamard linear (replaces _make_w8a8_hadamard_forward._forward,
 * src/zimage_triton/quantization/int8_linear.py:114-138)
 * ------------------------------------------------------------------------- */

/* Activation rotation + per-token int8 quantisation
 * (int8_linear.py:119-130; hadamard.py:78-107).
 * x: bf16 [M,K] row stride ldx; q: int8 [M,K] row stride ldq; sx: bf16 [M].
 * hadamard!=0 applies the block-128 Walsh-Hadamard rotation (K % 128 == 0);
 * hadamard==0 is the plain W8A8 quantisation (int8_linear.py:87-88).
 * x_rot (nullable): bf16 [M,K] stride ldq, the rotated activations (debug). */
ZIB_API int zib_act_quant(const void* x, int64_t ldx, void* q, int64_t ldq, void* sx,
                  void* x_rot, int64_t M, int64_t K, int hadamard, void* stream);

/* int8 GEMM + dequant epilogue on tcgen05 tensor cores
 * (torch._int_mm + epilogue, int8_linear.py:133-137):
 *   y[m,n] = bf16( bf16(acc) * bf16(sx[m]*sw[n]) ) (+ bias[n], bf16 add)
 *   acc[m,n] = sum_k q[m,k] * wq[n,k]   (int32, exact)
 * q: int8 [M,K] stride ldq; wq: int8 [N,K] stride ldw (nn.Linear layout);
 * sx: bf16 [M]; sw: bf16 [N]; bias: bf16 [N] or NULL; y: bf16 [M,N] stride ldy.
 * Requires K % 16 == 0, ldq/ldw % 16 == 0, ldy % 8 == 0, 16-byte aligned bases. */
ZIB_API int zib_gemm_w8a8(const void* q, int64_t ldq, const void* wq, int64_t ldw,
                  const void* sx, const void* sw, const void* bias,
                  void* y, int64_t ldy, int64_t M, int64_t N, int64_t K, void* stream);

/* Same GEMM writing the raw int32 accumulators (debug / bit-exactness checks of
 * torch._int_mm, int8_linear.py:133).  acc: int32 [M,N] stride ldacc (% 4 == 0). */
ZIB_API int zib_gemm_w8a8_acc_i32(const void* q, int64_t ldq, const void* wq, int64_t ldw,
                          void* acc, int64_t ldacc, int64_t M, int64_t N, int64_t K,
                          void* stream);

/* FFN up-projection with the SwiGLU and the w2-input rotation fused into the
 * GEMM epilogue.  Replaces, in one launch, the two int8 linears w1/w3
 * (int8_linear.py:133-137), swiglu_fwd (kernels/swiglu.py:51-58: silu(g)
 * rounded to bf16, times u, rounded to bf16) and the block-128 Hadamard
 * rotation of the w2 input (int8_linear.py:119-126, hadamard.py:78-107):
 *   g = dequant(q.w1^T), u = dequant(q.w3^T)                 (bf16 [M,F])
 *   x_rot[m, 128j:128j+128] = bf16( H128 . bf16(bf16(silu(g)) * u) ) * bf16(1/sqrt(128))
 * q: int8 [M,K] stride ldq; w1, w3: int8 [F,K] stride ldw; sx: bf16 [M];
 * sw1, sw3: bf16 [F]; x_rot: bf16 [M,F] stride ldo.  F % 128 == 0.
 * x_rot is what zib_act_quant(..., hadamard=0) quantises for w2. */
ZIB_API int zib_gemm_w8a8_swiglu_had(const void* q, int64_t ldq, const void* w1, const void* w3,
                             int64_t ldw, const void* sx, const void* sw1, const void* sw3,
                             void* x_rot, int64_t ldo, int64_t M, int64_t F, int64_t K,
                             void* stream);

/* zib_gemm_w8a8_swiglu_had with w1 and w3 as the two halves of one int8 [2F, K]
 * tensor (row stride ldw): rows 0..F-1 = w1, rows F..2F-1 = w3, i.e. the
 * two-weight call with w3 = w13 + F * ldw.  Each CTA then stages its 64 rows of
 * each weight per k-block with one 3-D TMA copy instead of two.  Same
 * arithmetic and output, bit for bit; w1 and w3 stay usable as the [F, K]
 * halves.  Same reference interfaces as zib_gemm_w8a8_swiglu_had (a layout of
 * the prepared weights, no reference counterpart of its own). */
ZIB_API int zib_gemm_w8a8_swiglu_had_w13(const void* q, int64_t ldq, const void* w13, int64_t ldw,
                                 const void* sx, const void* sw1, const void* sw3, void* x_rot,
                                 int64_t ldo, int64_t M, int64_t F, int64_t K, void* stream);

/* QKV projection with the per-head Q/K RMSNorm and the interleaved RoPE fused
 * into the GEMM epilogue.  Replaces the int8 qkv linear (int8_linear.py:133-137)
 * followed by fused_qknorm_rope on Q and K (kernels/fused_qknorm_rope.py:85-151).
 * y: bf16 [M, 3*heads*128] stride ldy holding [Q | K | V] (head_dim 128, rows
 * are (batch, token) with seq tokens per batch entry), Q and K normalised with
 * q_norm_w/k_norm_w (fp32 [128], eps q_eps/k_eps) and rotated with the
 * fp32 cos/sin tables [B][seq][64] (batch stride cs_b, 0 when shared); V is the
 * plain dequantised projection.  heads even, M % seq == 0. */
ZIB_API int zib_gemm_w8a8_qk_norm_rope(const void* q, int64_t ldq, const void* wq, int64_t ldw,
                               const void* sx, const void* sw, void* y, int64_t ldy,
                               int64_t M, int64_t N, int64_t K,
                               const float* q_norm_w, const float* k_norm_w, float q_eps,
                               float k_eps, const float* cos, const float* sin, int64_t cs_b,
                               int64_t seq, int64_t heads, void* stream);

/* Selects the GEMM tiling for subsequent zib_gemm_w8a8* calls on this process:
 * 0 = automatic (2-CTA 256x256 tiles with cta_group::2 when M > 128, 1-CTA
 * 128x256 tiles for 9-128 rows, and for the plain and int32 entry points a
 * dp4a kernel that streams the weights when M <= 8 and K <= 4096), 1 = always
 * 1-CTA, 2 = always 2-CTA.  Results are bit-identical across variants.  No
 * reference counterpart (tuning knob). */
ZIB_API int zib_gemm_set_variant(int variant);

/* Split-K tail for zib_gemm_w8a8 and zib_gemm_w8a8_acc_i32 with 2-CTA tiles
 * (on by default): when the last wave of tiles is short and K >= 6144, its
 * tiles run as 2-4 units over slices of K whose int32 partials are summed by
 * the last unit to finish (bit-identical results).  It needs the workspace
 * that the caller registers with zib_gemm_set_split_workspace; without one
 * the GEMM runs unsplit.  The same switch governs the half-width tail: a last
 * wave of at most half as many tiles as CTA pairs (and no split) runs as twice
 * as many units of 128 output columns.  No reference counterpart (tuning knob). */
ZIB_API int zib_gemm_set_split(int enable);

/* L2 budget of the GEMM tile order for subsequent zib_gemm_w8a8* calls on this
 * process, in bytes (0 restores the default, 48 MiB): the operand that every
 * wave of concurrent tiles re-reads is swept in groups of blocks whose rows fit
 * the budget, all tiles of one group before the next.  Results are identical
 * for every budget.  No reference counterpart (tuning knob). */
ZIB_API int zib_gemm_set_group_budget(int64_t bytes);

/* Registers the caller's split-K workspace for `device` (NULL, NULL
 * unregisters): `ws` (16-byte aligned) holds ws_bytes / 256 KB partial-tile
 * pairs, `counters` n_counters int32 that must be zero when registered (each
 * completed GEMM leaves them at zero; zib_device_error_read_clear() re-zeroes
 * them after a device error).  The caller keeps both alive while GEMMs may use
 * them, and GEMMs on that device that use them must not overlap on the GPU.
 * One 256 KB pair per two SMs and two counters per pair cover every launch
 * (~19 MB on B200).  No reference counterpart (the caller owns all workspaces). */
ZIB_API int zib_gemm_set_split_workspace(int device, void* ws, int64_t ws_bytes, void* counters,
                               int64_t n_counters);

/* zib_gemm_w8a8 for callers that must not allocate device memory: a host
 * framework that owns the GPU's memory through its own pool and budget (a
 * cudaMalloc behind its back fragments the pool, escapes its accounting and
 * can fail when the pool already holds the free memory), code recording a CUDA
 * stream capture (which refuses cudaMalloc), and latency-bound loops (cudaMalloc
 * and cudaFree synchronise the device).  Its split-K tail uses a static device
 * scratch area instead of a workspace that the caller would have to allocate
 * and register (zib_gemm_set_split_workspace); the call allocates and frees
 * nothing.  `splits` (1-4, and at most ceil(K / 128), the number of 128-wide
 * K-blocks) is the number of K-slices each tile of a short last wave runs as
 * (2-CTA tiles, M > 128; 1 = no split; launches without a short last wave run
 * unsplit); more splits than K-blocks returns ZIB_ERR_INVALID_ARG.  Limit: the
 * scratch holds 64 units of 256 KB (16 MB of device memory on every GPU that
 * loads this library, held until the process exits) and 128 arrival counters;
 * a call whose last wave needs more (its tiles x splits > 64) returns
 * ZIB_ERR_TOO_LARGE before launching.  The counters must start at zero: they
 * do (static initialisation), every completed call leaves them at zero, and
 * zib_device_error_read_clear() re-zeroes them after a device error.  The
 * first call on each device looks up the scratch address with
 * cudaGetSymbolAddress (with that device current) and should come before any
 * stream capture.  Every call shares the scratch: calls that overlap on the GPU
 * (any streams of one device) race.  No counterpart in the reference. */
ZIB_API int zib_gemm_w8a8_static_scratch(const void* q, int64_t ldq, const void* wq, int64_t ldw,
                               const void* sx, const void* sw, const void* bias, void* y,
                               int64_t ldy, int64_t M, int64_t N, int64_t K, int splits,
                               void* stream);

/* Offline weight prep: rotate_weight (hadamard.py:47-75) in exact arithmetic
 * rounded to fp32, then _quantize_weight_per_channel (int8_linear.py:67-73).
 * w: bf16 [N,K] stride ldw -> wq int8 [N,K] stride ldq, sw bf16 [N]
 * (the `_w_scale` buffer), sw_f32 fp32 [N] (nullable), w_rot fp32 [N,K]
 * stride ld_rot (nullable: the rotated weight itself).  hadamard as above. */
ZIB_API int zib_weight_prep(const void* w, int64_t ldw, void* wq, int64_t ldq, void* sw,
                    void* sw_f32, float* w_rot, int64_t ld_rot, int64_t N, int64_t K,
                    int hadamard, void* stream);

/* ---------------------------------------------------------------------------
 * Bandwidth-bound row kernels (replace the Triton kernels)
 * ------------------------------------------------------------------------- */

/* RMSNorm: y = bf16(bf16(x*rstd)*w) (kernels/rms_norm.py:18-59, :62-102).
 * x, y: bf16 [rows, n] strides ldx/ldy; w: fp32 [n]. */
ZIB_API int zib_rms_norm(const void* x, int64_t ldx, const float* w, void* y, int64_t ldy,
                 int64_t rows, int64_t n, float eps, void* stream);

/* RMSNorm + adaLN modulation, bf16 output (rms_norm.py:47-57 then
 * patching_comfyui.py:378/:401): y = bf16( rmsnorm(x) * bf16(1 + scale[b]) )
 * (+ shift[b] if shift != NULL).  scale/shift: bf16 rows of length n with row
 * stride ld_mod, batch index b = row / rows_per_batch. */
ZIB_API int zib_rmsnorm_mod(const void* x, int64_t ldx, const float* w, const void* scale,
                    const void* shift, int64_t ld_mod, int64_t rows_per_batch,
                    void* y, int64_t ldy, int64_t rows, int64_t n, float eps, void* stream);

/* RMSNorm + adaLN modulation fused with the next W8A8 linear's activation
 * rotation + quantisation (same math as zib_rmsnorm_mod followed by
 * zib_act_quant).  q int8 [rows,n] stride ldq, sx bf16 [rows]. */
ZIB_API int zib_rmsnorm_mod_quant(const void* x, int64_t ldx, const float* w, const void* scale,
                          const void* shift, int64_t ld_mod, int64_t rows_per_batch,
                          void* q, int64_t ldq, void* sx, int64_t rows, int64_t n,
                          float eps, int hadamard, void* stream);

/* Fused RMSNorm + gate + residual (kernels/fused_norm_residual.py:23-74, :77-126):
 * y = bf16( r + bf16( gate[b] * bf16(bf16(x*rstd)*w) ) ); gate: bf16 rows
 * (stride ld_gate) indexed by b = row / rows_per_batch (no expand copy). */
ZIB_API int zib_norm_gate_residual(const void* x, int64_t ldx, const void* r, int64_t ldr,
                           const void* gate, int64_t ld_gate, int64_t rows_per_batch,
                           const float* w, void* y, int64_t ldy, int64_t rows, int64_t n,
                           float eps, void* stream);

/* zib_norm_gate_residual fused with the following RMSNorm + modulation +
 * W8A8 activation quantisation (patching_comfyui.py:386-401 then
 * int8_linear.py:119-130): writes y (the new residual stream) and q/sx of
 * bf16(rmsnorm(y; w2) * bf16(1 + scale[b])) (+ shift). */
ZIB_API int zib_norm_gate_residual_mod_quant(const void* x, int64_t ldx, const void* r, int64_t ldr,
                                     const void* gate, int64_t ld_gate, int64_t rows_per_batch,
                                     const float* w, void* y, int64_t ldy,
                                     const float* w2, const void* scale, const void* shift,
                                     int64_t ld_mod, void* q, int64_t ldq, void* sx,
                                     int64_t rows, int64_t n, float eps, float eps2,
                                     int hadamard, void* stream);
/* zib_norm_gate_residual_mod_quant with the norm weights w, w2 given as bf16 (the
 * modules' own bf16 parameters) instead of fp32 copies: the same results for the same
 * weight values (the product of a bf16 weight and a bf16 value is exact in fp32 in the
 * normal range, so one bf16 rounding of it equals the fp32 product rounded to bf16),
 * half the weight traffic.  Rows of n = 3840 features only; ZIB_ERR_INVALID_ARG
 * otherwise.  Same reference lines as above. */
ZIB_API int zib_norm_gate_residual_mod_quant_w16(const void* x, int64_t ldx, const void* r, int64_t ldr,
                                         const void* gate, int64_t ld_gate, int64_t rows_per_batch,
                                         const void* w, void* y, int64_t ldy,
                                         const void* w2, const void* scale, const void* shift,
                                         int64_t ld_mod, void* q, int64_t ldq, void* sx,
                                         int64_t rows, int64_t n, float eps, float eps2,
                                         int hadamard, void* stream);

/* SwiGLU: out = bf16( bf16(silu_fp32(gate)) * up ) (kernels/swiglu.py:20-59, :62-110).
 * gate/up/out: bf16 [rows, n] with strides ldg/ldu/ldo. */
ZIB_API int zib_swiglu(const void* gate, int64_t ldg, const void* up, int64_t ldu, void* out,
               int64_t ldo, int64_t rows, int64_t n, void* stream);

/* SwiGLU fused with the down projection's activation rotation + quantisation
 * (swiglu.py:51-58 then int8_linear.py:119-130). */
ZIB_API int zib_swiglu_quant(const void* gate, int64_t ldg, const void* up, int64_t ldu,
                     void* q, int64_t ldq, void* sx, int64_t rows, int64_t n,
                     int hadamard, void* stream);

/* Fused per-head RMSNorm + interleaved-pair RoPE
 * (kernels/fused_qknorm_rope.py:38-151, :154-235), or RoPE alone when
 * w == NULL (kernels/rope_3d.py:22-89, :92-163).
 * x/out: bf16 [B,S,H,d] with element strides (sb, ss, sh), last dim contiguous
 * (out may alias x); cos/sin: fp32 [Bf,S,d/2] contiguous per batch with batch
 * stride cs_b (0 = shared across batch); w: fp32 [d] or NULL.  d == 128. */
ZIB_API int zib_qknorm_rope(const void* x, int64_t x_sb, int64_t x_ss, int64_t x_sh,
                    void* out, int64_t o_sb, int64_t o_ss, int64_t o_sh,
                    const float* cos, const float* sin, int64_t cs_b,
                    const float* w, int64_t B, int64_t S, int64_t H, int64_t d,
                    float eps, void* stream);

/* adaLN modulation, Triton variant (kernels/adaln_modulation.py:28-88, :91-155):
 * raw bf16 [rows, 4*dim] stride ldr -> (1+scale_msa, tanh(gate_msa),
 * 1+scale_mlp, tanh(gate_mlp)), each bf16 [rows, dim] contiguous. */
ZIB_API int zib_adaln_modulation(const void* raw, int64_t ldr, void* scale_msa, void* gate_msa,
                         void* scale_mlp, void* gate_mlp, int64_t rows, int64_t dim,
                         void* stream);

/* Gates of the eager default path (patching_comfyui.py:368-372): from raw bf16
 * [rows, 4*dim], writes tanh(gate_msa) and tanh(gate_mlp) into gates
 * bf16 [rows, 2, dim] contiguous. */
ZIB_API int zib_adaln_gates(const void* raw, int64_t ldr, void* gates, int64_t rows, int64_t dim,
                    void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ZIMAGE_B200_H_ */
