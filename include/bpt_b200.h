/* bpt_b200: the decode hot path of fastserve / nanoserve (ish-codes-magic/bytes-per-token), as sm_100a CUDA
 * kernels behind a plain C ABI.
 *
 * Conventions
 *  - Every entry point is `extern "C"`, takes plain device pointers, sizes and strides (in elements) and a
 *    cudaStream_t (passed as void*; NULL is the legacy default stream), launches asynchronously, and returns a
 *    status: 0 on success, a BPT_ERR_* code otherwise. bpt_last_error() gives the message of the last failure
 *    on the calling host thread. Nothing here allocates device memory, synchronizes, or reads device memory
 *    on the host, so every launch can be captured in a CUDA graph.
 *  - The caller owns all memory: inputs, outputs and workspaces. Kernels never trap: a device-side problem
 *    (a block-table entry out of range, a bounded wait that ran out) is recorded in a device flag that
 *    bpt_device_error() reads (that call synchronizes the device) and the offending data is skipped.
 *  - Shapes use B sequences, Hq query heads, Hkv KV heads, D head dim, S splits, M tokens, N outputs,
 *    K inputs.
 *
 * Each function names the reference interface it replaces (paths inside the reference project).
 */
#ifndef BPT_B200_H_
#define BPT_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BPT_ABI_VERSION 1

/* status codes */
#define BPT_OK 0
#define BPT_ERR_INVALID 1     /* a shape, stride, dtype or pointer argument is wrong            -> ValueError   */
#define BPT_ERR_UNSUPPORTED 2 /* a valid configuration this build has no kernel for             -> ValueError   */
#define BPT_ERR_ALIGNMENT 3   /* a pointer or stride breaks the 16-byte rule of the bulk copies -> ValueError   */
#define BPT_ERR_WORKSPACE 4   /* the workspace given is smaller than required                   -> ValueError   */
#define BPT_ERR_CUDA 5        /* the CUDA runtime reported an error at launch                   -> RuntimeError */

/* element types */
#define BPT_DTYPE_F32 0
#define BPT_DTYPE_F16 1
#define BPT_DTYPE_BF16 2

/* KV cache formats */
#define BPT_KV_FP8 1  /* E4M3 bytes, one fp32 scale per tensor (K and V each)            */
#define BPT_KV_INT8 2 /* symmetric int8 codes, one fp16 scale per (token, KV head)      */

/* launch flags */
#define BPT_FLAG_PDL 1 /* launch with programmatic dependent launch (prologue overlaps the previous kernel) */
/* With BPT_FLAG_PDL, for the paged attention: the caller promises that the lengths, the block table and the KV
 * pools are not written by the kernel this launch follows, so the kernel maps its pages and starts their copies
 * before it waits on that kernel (q, the output and the workspace are still touched only after the wait). */
#define BPT_FLAG_KV_READY 2
/* For tests of the bounded device waits only. One CTA of the launch (the one holding the first page, or the first
 * weight tile) stops issuing its copies partway (every copy it did issue is still awaited, so nothing is left in
 * flight), the waits that then find no data give up after
 * ~2 ms instead of ~200 ms, the call records device error 1 (a bounded wait ran out; bpt_device_error) and its
 * outputs are undefined. Taken by bpt_paged_attend / bpt_paged_attend_noalloc where they run the persistent kernel
 * (it turns BPT_FLAG_KV_READY off) and by bpt_w4a16_linear / bpt_w4a16_gate_up_silu where they run the tcgen05
 * GEMM; every other launch ignores it. */
#define BPT_FLAG_TEST_STALL 0x40000000

int bpt_abi_version(void);
const char* bpt_last_error(void);
/* Synchronizes the device, returns the first device-side error code recorded since the last call and clears
 * it (0 = none, 1 = a bounded wait ran out, 2 = a block-table entry out of range, 3 = a slot out of range). */
int bpt_device_error(void);

/* ---- W4A16: INT4 group-wise weight-only linear ---------------------------------------------------------------
 * y[M, N] = x[M, K] . W^T, W[n, k] = scale[n, g] * (q[n, k] - zero[n, g]), g = k / group, fp32 accumulation,
 * y rounded once to bf16.
 *   x        bf16 [M, K], row stride ldx
 *   qweight  int32 [N, K/8]: code k of row n at bits 4(k mod 8) of word k/8, unsigned 0..15
 *   scales   fp16 [N, K/group]
 *   qzeros   int32 [N, ceil(K/group/8)]: zero-point g of row n at bits 4(g mod 8) of word g/8, or NULL for
 *            compressed-tensors' symmetric layout (an implicit zero-point of 8)
 *   y        bf16 [M, N], row stride ldy
 * group a multiple of 32 dividing K; qweight 16-byte aligned.
 * Replaces: nn.Linear on a dequantized weight (src/fastserve/engine/model.py:43-46, :91-96) fed by
 * quant/compressed.py:56-69 (dequantize_linear) and quant/rtn.py:103-114 (the asymmetric grid); in
 * production, vLLM's Marlin W4A16 kernel (docs/gates/M4-report.md:38-43). */
int bpt_w4a16_linear(const void* x, int64_t ldx, const int32_t* qweight, const void* scales, const int32_t* qzeros,
                     void* y, int64_t ldy, int64_t M, int64_t N, int64_t K, int64_t group, int flags, void* stream);

/* Fused gate_up + SwiGLU: the weight holds gate and up rows interleaved (row 2i = gate_proj row i,
 * row 2i+1 = up_proj row i; N = 2I rows), and y[M, I] = silu(x.Wg^T) * (x.Wu^T), computed from the fp32 sums.
 * Replaces: MLP.gate_proj / up_proj and silu(g) * u (src/fastserve/engine/model.py:91-96), the shared-input
 * group "gate_up" of quant/equivalence.py:40. */
int bpt_w4a16_gate_up_silu(const void* x, int64_t ldx, const int32_t* qweight, const void* scales,
                           const int32_t* qzeros, void* y, int64_t ldy, int64_t M, int64_t N, int64_t K,
                           int64_t group, int flags, void* stream);

/* Which kernel bpt_w4a16_linear / bpt_w4a16_gate_up_silu launch for a shape (given 16-byte aligned scales and zero
 * points), and so which arithmetic produces y:
 *   BPT_W4A16_KERNEL_TCGEN05    M >= 16: the dense bf16 weight round_bf16(scale * (q - zero)) (one rounding, as
 *                               quant/compressed.py:56-69 builds it) contracted on the tcgen05 tensor cores, fp32
 *                               accumulation;
 *   the others                  every group's sum of x (q - zero) in fp32, times the fp32 scale (no weight rounding).
 * Returns a BPT_W4A16_KERNEL_* value. */
#define BPT_W4A16_KERNEL_CUDA_CORES 0
#define BPT_W4A16_KERNEL_MMA_GEMV 1
#define BPT_W4A16_KERNEL_STREAM 2
#define BPT_W4A16_KERNEL_MMA_GEMM 3
#define BPT_W4A16_KERNEL_TCGEN05 4
int bpt_w4a16_kernel(int64_t M, int64_t N, int64_t K, int64_t group, int has_zeros);

/* RTN-quantize a dense weight W [N, K] (bf16 or fp32, row-major) to the W4A16 format above: per group of
 * `group` inputs, scale = fp16((max(w,0) - min(w,0)) / 15) (1.0 for an all-zero group), zero =
 * round(-min / scale), code = clamp(round(w / scale) + zero, 0, 15), rounding half to even.
 * Replaces: quant/rtn.py:77-92,107-114 (scale_and_zero / quantize, asymmetric) with the fp16-scale-first
 * convention of kernels/reference.py:103-114, and the int32 packing of quant/compressed.py:25-41. */
int bpt_w4a16_quantize(const void* w, int w_dtype, int64_t N, int64_t K, int64_t group, int32_t* qweight,
                       void* scales, int32_t* qzeros, void* stream);

/* ---- paged decode attention over an FP8 / INT8 KV cache --------------------------------------------------------
 * One query token per sequence. Pools are [num_blocks, block_size, Hkv, D] (engine/kv_cache.py:108), one
 * byte per element; block_table int32 [B, bt_stride] maps logical block j of sequence b to its physical block;
 * lengths int32 [B]: sequence b attends to its first lengths[b] tokens. KV head h serves query heads
 * h*REP .. h*REP+REP-1 (REP = Hq/Hkv), as engine/attention.py:23-31.
 *   q            [B, Hq, D] of q_dtype, strides (q_stride_b, q_stride_h), unit stride over D
 *   kind         BPT_KV_FP8: k_scale_f32 / v_scale_f32 are the per-tensor scales, k_scales/v_scales unused
 *                BPT_KV_INT8: k_scales / v_scales are fp16 [num_blocks, block_size, Hkv]
 *   split        tokens per split, a multiple of block_size; n_splits >= ceil(max length / split)
 *   sm_scale     the softmax scale (head_dim^-0.5 in the model)
 * Supported: D in {64, 128, 256}, REP in {1, 2, 4, 8}, Hkv <= 16, block_size in {8, 16, 32}; pools and every
 * page 16-byte aligned.
 */

/* Per-split partial attentions: out_partial f32 [B, Hq, n_splits, D] and lse_partial f32 [B, Hq, n_splits]
 * (log-sum-exp of the split's scores; a split with no token has out 0, lse -inf).
 * Replaces: kernels/kv_attention.py:190-245 (decode_attention) for a paged cache; the per-split contract of
 * kv_attention.py:167-173 and kernels/reference.py:186-202 (partial_attention). */
int bpt_paged_decode_partials(const void* q, int q_dtype, int64_t q_stride_b, int64_t q_stride_h,
                              const void* k_pool, const void* v_pool, int kind, float k_scale_f32,
                              float v_scale_f32, const void* k_scales, const void* v_scales,
                              const int32_t* block_table, int64_t bt_stride, const int32_t* lengths, int64_t B,
                              int64_t Hq, int64_t Hkv, int64_t D, int64_t block_size, int64_t num_blocks,
                              int64_t split, int64_t n_splits, float sm_scale, float* out_partial,
                              float* lse_partial, int flags, void* stream);

/* The merged attention out [B, Hq, D] in out_dtype, splits merged inside the same launch: the last CTA of a
 * sequence to finish combines its splits (an atomic ticket per sequence; nothing waits). `workspace` is
 * caller-owned device memory of at least bpt_paged_attend_workspace_bytes(...) bytes, ZEROED before its
 * first use; its first 256 KiB hold the per-sequence tickets (B <= 65536), which every call leaves at zero
 * again, so one workspace serves calls of any shape. Calls that share a workspace must not overlap.
 * Replaces: kernels/kv_attention.py:248-252 (attend = merge_partials(decode_attention(...))) and
 * kernels/reference.py:205-211 (merge_partials). */
int64_t bpt_paged_attend_workspace_bytes(int64_t B, int64_t Hq, int64_t D, int64_t n_splits);
int bpt_paged_attend(const void* q, int q_dtype, int64_t q_stride_b, int64_t q_stride_h, const void* k_pool,
                     const void* v_pool, int kind, float k_scale_f32, float v_scale_f32, const void* k_scales,
                     const void* v_scales, const int32_t* block_table, int64_t bt_stride, const int32_t* lengths,
                     int64_t B, int64_t Hq, int64_t Hkv, int64_t D, int64_t block_size, int64_t num_blocks,
                     int64_t split, int64_t n_splits, float sm_scale, void* out, int out_dtype, void* workspace,
                     int64_t workspace_bytes, int flags, void* stream);

/* bpt_paged_attend without a workspace argument, for callers that cannot allocate device memory: serving
 * engines that hand all free HBM to their paged KV pool at start-up (so a later cudaMalloc fails or fragments
 * the pool), runtimes whose memory policy forbids device allocation after initialization, and foreign-language
 * hosts that only hold the buffers they were given and have no allocator to call. No counterpart in the
 * reference (its attention allocates its partial outputs with torch.empty on every call).
 * The split partials and tickets live in one fixed array of BPT_NOALLOC_SCRATCH_BYTES bytes, a static device
 * variable of this library: every GPU that loads the library holds it until the process exits. A call needs
 * 256 KiB + S * Hq * (D + 1) * 4 bytes of it (rounded up to 256 B per part), S = B + the GPU's SM count for
 * contiguous q with D 64 or 128 and Hkv <= 8, S = B * n_splits otherwise, and returns BPT_ERR_WORKSPACE,
 * launching nothing, when that is more. The array used is the current device's: q (and every other tensor) must be
 * memory of the current device (BPT_ERR_INVALID otherwise). The first call on a device looks up the array's
 * device address (cudaGetSymbolAddress) with that device current, and looks it up again when the device's current
 * context has changed (after a cudaDeviceReset, say); make that first call before any stream capture. Each call
 * clears the tickets it uses (an asynchronous memset on `stream`) before the kernel, so BPT_FLAG_PDL and
 * BPT_FLAG_KV_READY give no overlap with the previous kernel here (the memset sits between them).
 * All calls on a device share the array: calls that overlap on the GPU (concurrent streams) race and corrupt
 * each other's results. Nothing here calls cudaMalloc, cudaFree or any allocating routine. */
#define BPT_NOALLOC_SCRATCH_BYTES (16 * 1024 * 1024)
int bpt_paged_attend_noalloc(const void* q, int q_dtype, int64_t q_stride_b, int64_t q_stride_h, const void* k_pool,
                             const void* v_pool, int kind, float k_scale_f32, float v_scale_f32, const void* k_scales,
                             const void* v_scales, const int32_t* block_table, int64_t bt_stride,
                             const int32_t* lengths, int64_t B, int64_t Hq, int64_t Hkv, int64_t D, int64_t block_size,
                             int64_t num_blocks, int64_t split, int64_t n_splits, float sm_scale, void* out,
                             int out_dtype, int flags, void* stream);

/* merged[B, Hq, D] (out_dtype) = sum_s softmax_s(lse[b, h, :]) * outs[b, h, s, :]; all -inf rows give 0.
 * Replaces: kernels/reference.py:205-211 (merge_partials). */
int bpt_merge_partials(const float* outs, const float* lses, int64_t B, int64_t Hq, int64_t S, int64_t D,
                       void* merged, int out_dtype, void* stream);

/* ---- KIVI contiguous decode attention (the reference's own cache layout) -----------------------------------
 * The QuantKV layout of kernels/reference.py:66-100: bits 4 or 8: uint8 codes k_codes/v_codes
 * [B, Hkv, t_max, D] (bits 8) or [B, Hkv, t_max, D/2] (bits 4, channel d low nibble / d + D/2 high nibble),
 * k_scale/k_zero fp16 [B, Hkv, n_groups, D] (one grid per channel per `group` tokens), v_scale/v_zero fp16
 * [B, Hkv, t_max] (one grid per token); bits 16: k_codes/v_codes are the keys and values themselves in
 * code_dtype and the grids are unused. Writes out_partial f32 [B, Hq, n_splits, D], lse_partial f32
 * [B, Hq, n_splits]; split is a multiple of group.
 * Supported: D in {16, 32, 64, 128, 256}, REP in {1, 2, 4, 8}, group 32.
 * Replaces: kernels/kv_attention.py:55-175 (the Triton kernel) behind decode_attention (:190-245). */
int bpt_kivi_decode_partials(const void* q, int q_dtype, int64_t q_stride_b, int64_t q_stride_h, int bits,
                             int code_dtype, const void* k_codes, const void* v_codes, const void* k_scale,
                             const void* k_zero, const void* v_scale, const void* v_zero, const int32_t* lengths,
                             int64_t B, int64_t Hq, int64_t Hkv, int64_t D, int64_t t_max, int64_t n_groups,
                             int64_t group, int64_t split, int64_t n_splits, float sm_scale, float* out_partial,
                             float* lse_partial, void* stream);

/* ---- the quantized KV write path ---------------------------------------------------------------------------------
 * Quantize k, v [B, Hkv, Q, D] (in_dtype; strides in elements for b, h, q; unit stride over D) and scatter token
 * (b, i) to slot write_offsets[b, i] of block write_blocks[b, i] (int32 [B, Q], row stride Q).
 * BPT_KV_FP8: code = e4m3(clamp(x / scale, -448, 448)), round to nearest even.
 * BPT_KV_INT8: scale = fp16(max|x| / 127) (1.0 for an all-zero vector), code = clamp(round(x / scale), -128, 127);
 * the scale goes to k_scales/v_scales[block, slot, h].
 * Replaces: PagedKVCache.update's write (engine/kv_cache.py:150-161) with kv/quant.py:40-48 (store) in front,
 * and QuantizedKVCache._append (integration/kv_cache.py:139-158) for a paged cache. */
int bpt_paged_kv_write(const void* k, const void* v, int in_dtype, int64_t stride_b, int64_t stride_h,
                       int64_t stride_q, int64_t B, int64_t Hkv, int64_t Q, int64_t D, const int32_t* write_blocks,
                       const int32_t* write_offsets, void* k_pool, void* v_pool, int kind, float k_scale_f32,
                       float v_scale_f32, void* k_scales, void* v_scales, int64_t block_size, int64_t num_blocks,
                       void* stream);

/* KIVI quantization of whole key groups: k, v [B, Hkv, T, D] (in_dtype, contiguous), T a multiple of group,
 * written at token offset t0 of a QuantKV cache with t_max tokens and n_groups grids (t0 a multiple of group).
 * Replaces: kernels/reference.py:132-160 (quantize_kv) as called from integration/kv_cache.py:146-154. */
int bpt_kivi_quantize(const void* k, const void* v, int in_dtype, int64_t B, int64_t Hkv, int64_t T, int64_t D,
                      int bits, int64_t group, void* k_codes, void* v_codes, void* k_scale, void* k_zero,
                      void* v_scale, void* v_zero, int64_t t_max, int64_t n_groups, int64_t t0, void* stream);

/* ---- the decode step's ops around the hot path (the caller side: config 5's Qwen3 step) -------------------------
 * bf16 tensors, row-major. RMSNorm of engine/model.py:24-36 with the residual add of DecoderLayer.forward
 * (:109-111) in front: h' = bf16(h + delta) (delta NULL: h' = h), x = bf16(weight * bf16(h' * rsqrt(mean(h'^2) +
 * eps))), statistics in fp32; h' goes to h_out when h_out is not NULL. hidden a multiple of 8 up to 16384,
 * 16-byte aligned tensors. Replaces: RMSNorm.forward and the residual adds (engine/model.py:24-36, 109-111). */
int bpt_rms_norm_residual(const void* h, const void* delta, const void* weight, void* h_out, void* x_out,
                          int64_t rows, int64_t hidden, float eps, int flags, void* stream);

/* One new token per sequence, from the fused q/k/v projection qkv [B, ld] (q heads, then k heads, then v heads,
 * D = 128 each): q head -> RMSNorm(q_norm) -> rotate-half RoPE(cos, sin [B, D]) -> q_out [B, Hq, D]; k head ->
 * RMSNorm(k_norm) -> RoPE -> FP8 E4M3 store (x / k_scale, as bpt_paged_kv_write) at slot write_offsets[b] of block
 * write_blocks[b] of k_pool [num_blocks, block_size, Hkv, D]; v head -> FP8 store to v_pool. Every bf16 rounding
 * of the reference's tensors is kept. Replaces: Attention.forward's q_norm / k_norm and rope.apply
 * (engine/model.py:63-70, engine/rope.py:31-43) and the cache write (engine/kv_cache.py:150-161). */
int bpt_qk_norm_rope_kv_write(const void* qkv, int64_t ld, int64_t B, int64_t Hq, int64_t Hkv, int64_t D,
                              const void* q_norm, const void* k_norm, const void* cos, const void* sin, float eps,
                              void* q_out, const int32_t* write_blocks, const int32_t* write_offsets, void* k_pool,
                              void* v_pool, float k_scale, float v_scale, int64_t block_size, int64_t num_blocks,
                              int flags, void* stream);

/* RMSNorm fused with per-token symmetric INT8 quantization (the activation quantizer before a W8A8 linear):
 * for every row of x [rows, d] (x_dtype, row stride x_row_stride elements, unit inner stride) and weight [d]
 * (w_dtype), in fp32: y = x * (1 / sqrt(sum(x^2) / d + eps)) * weight, scale[row] = max(max|y| / 127, 1e-12),
 * codes[row] = clamp(rint(y / scale), -128, 127) -> codes int8 [rows, d] contiguous, scale float32 [rows].
 * delta (NULL for none): x + delta, rounded to x_dtype, is normalized instead and goes to x_out (NULL: not
 * written); delta and x_out are contiguous [rows, d] in x_dtype. Any d >= 1; 16-byte vector accesses when
 * alignment allows. Replaces: kernels/norm_quant.py:72-109 (rms_norm_int8, its Triton kernel :42-67), defined
 * by kernels/reference.py:44-55; with delta, also the residual add of engine/model.py:109-111. */
int bpt_rms_norm_int8(const void* x, int x_dtype, int64_t x_row_stride, const void* weight, int w_dtype,
                      const void* delta, void* x_out, void* codes, void* scale, int64_t rows, int64_t d, float eps,
                      int flags, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* BPT_B200_H_ */
